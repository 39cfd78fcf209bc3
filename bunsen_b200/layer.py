"""The gated DeltaNet layer's steps around the rule, on CUDA tensors, through
libgdr's C ABI (include/gdr.h):

* ``causal_conv1d`` -- bunsen's ``causal_depthwise_conv1d``
  (``ops/transformers/linear_attention/causal_conv.rs:36-69``), optionally
  with the layer's silu and its q / k / v channel split
  (``blocks/transformers/mixers/gated_delta_net.rs:396-420``);
* ``gated_norm`` -- ``GatedNorm`` (``gated_delta_net.rs:439-440``) on its own;
* ``state_reorder`` -- ``DeltaNetState::reorder`` (``state.rs:112-135``).

The gates and the gated norm run with the rule itself:
``GatedDeltaRule.chunked(..., gates=..., norm=...)``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .rule import _DTYPES, _ptr, _stream


def causal_conv1d(x, weight, state=None, *, cu_seqlens=None, silu=False, splits=None,
                  state_out=None, with_state=True):
    """x ``[B, T, C]`` (or packed ``[T_total, C]`` with ``cu_seqlens``),
    weight ``[C, K]`` in x's dtype, state ``[N, K - 1, C]`` f32 or None.

    Returns ``(outputs, next_state)``: ``outputs`` is the convolution ``[.., C]``
    or, with ``splits=(c0, c1)``, the three channel ranges ``[0, c0)``,
    ``[c0, c1)``, ``[c1, C)`` as separate contiguous tensors; ``next_state``
    ``[N, K - 1, C]`` f32 (None when ``with_state`` is False). ``state_out``
    may be ``state`` (updated in place)."""
    if x.device.type != "cuda":
        raise RuntimeError("libgdr runs on CUDA tensors only")
    if x.dtype not in _DTYPES or weight.dtype != x.dtype:
        raise TypeError("x and weight share one dtype, f32, bf16 or f16")
    packed = cu_seqlens is not None
    if x.dim() != (2 if packed else 3):
        raise ValueError("x is [B, T, C], or [T_total, C] with cu_seqlens")
    c, k = weight.shape
    if x.shape[-1] != c:
        raise ValueError(f"weight [C, K] = {tuple(weight.shape)} against x {tuple(x.shape)}")
    x, weight = x.contiguous(), weight.contiguous()
    lead = tuple(x.shape[:-1])
    n = (cu_seqlens.numel() - 1) if packed else x.shape[0]
    c0, c1 = (c, c) if splits is None else splits
    outs = [torch.empty(lead + (w,), dtype=x.dtype, device=x.device)
            for w in (c0, c1 - c0, c - c1)]
    if state is not None:
        if tuple(state.shape) != (n, k - 1, c):
            raise ValueError(f"the state is [N, K - 1, C] = {(n, k - 1, c)}")
        state = state.to(torch.float32).contiguous()
    if with_state and state_out is None:
        state_out = torch.empty((n, k - 1, c), dtype=torch.float32, device=x.device)
    if packed:
        cu_seqlens = cu_seqlens.to(device=x.device, dtype=torch.int32).contiguous()
    p = _lib.GdrConvParams(batch=0 if packed else x.shape[0],
                           seq_len=x.shape[0] if packed else x.shape[1],
                           n_seqs=n if packed else 0, channels=c, taps=k, split0=c0, split1=c1,
                           silu=int(silu), dtype=_DTYPES[x.dtype])
    status = _lib.load().gdr_causal_conv1d(
        ctypes.byref(p), x.data_ptr(), weight.data_ptr(), _ptr(state),
        *(o.data_ptr() if o.numel() else None for o in outs),
        _ptr(state_out) if with_state else None, _ptr(cu_seqlens), _stream(x.device))
    _lib.check("gdr_causal_conv1d", status)
    return (outs[0] if splits is None else tuple(outs)), (state_out if with_state else None)


def gated_norm(x, z, weight, eps, out=None):
    """bunsen's ``GatedNorm`` (``gated_delta_net.rs:439-440``): ``rmsnorm(x) *
    weight * silu(z)`` over the last axis; x and z share shape and dtype;
    ``out`` may be ``x``."""
    if x.device.type != "cuda":
        raise RuntimeError("libgdr runs on CUDA tensors only")
    if x.dtype not in _DTYPES or z.dtype != x.dtype or z.shape != x.shape:
        raise TypeError("x and z share one shape and one dtype, f32, bf16 or f16")
    x, z = x.contiguous(), z.contiguous()
    weight = weight.to(torch.float32).contiguous()
    if out is None:
        out = torch.empty_like(x)
    width = x.shape[-1]
    status = _lib.load().gdr_gated_norm(x.numel() // width if width else 0, width, x.data_ptr(),
                                        z.data_ptr(), weight.data_ptr(), float(eps),
                                        _DTYPES[x.dtype], out.data_ptr(), _stream(x.device))
    _lib.check("gdr_gated_norm", status)
    return out


def state_reorder(src, sources, out=None):
    """Row ``r`` of the result is row ``sources[r]`` of ``src`` (any trailing
    shape, rows along dim 0); ``sources`` int32 on the device."""
    if src.device.type != "cuda":
        raise RuntimeError("libgdr runs on CUDA tensors only")
    src = src.contiguous()
    sources = sources.to(device=src.device, dtype=torch.int32).contiguous()
    rows = sources.numel()
    if out is None:
        out = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row_bytes = src[0].numel() * src.element_size() if src.shape[0] else 0
    status = _lib.load().gdr_state_reorder(src.data_ptr(), out.data_ptr(), sources.data_ptr(),
                                           rows, src.shape[0], row_bytes, _stream(src.device))
    _lib.check("gdr_state_reorder", status)
    return out
