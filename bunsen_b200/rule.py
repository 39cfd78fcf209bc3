"""``GatedDeltaRule`` over libgdr: the host-side mirror of bunsen's Rust
operator (``crates/public/bunsen/src/ops/transformers/linear_attention/
delta_rule.rs:51-310``), on CUDA tensors.

Same options (``qk_l2norm_eps``, ``chunk_size``), same argument order and
meaning (``q, k, v, g, beta, state``), same returns (the output in ``q``'s
dtype and the f32 state after the last position), and the same failures: a
shape that breaks bunsen's contracts (``delta_rule.rs:135-150``) or a zero
chunk (``:233``) raises before anything launches. Two extensions, both
opt-in: ``q`` and ``k`` may carry fewer heads than ``v`` (value head ``h``
reads key head ``h // (H_v // H_qk)``, the arithmetic of the
``repeat_interleave`` bunsen's caller applies, ``gated_delta_net.rs:404-419``),
and a packed ragged batch ``[T_total, H, .]`` with ``cu_seqlens``.

f64 inputs compute in f64, g, beta and the state included, as bunsen does
when its inputs are f64 (``burner/tensor/widening.rs:58-60``); the other
dtypes return an f32 state.

Every call runs a CUDA kernel of ``libgdr.so``; there is no other path.
"""

from __future__ import annotations

import ctypes
import dataclasses

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.GDR_DTYPE_F32, torch.bfloat16: _lib.GDR_DTYPE_BF16,
           torch.float16: _lib.GDR_DTYPE_F16}
_ALGOS = {"auto": _lib.GDR_ALGO_AUTO, "cuda_core": _lib.GDR_ALGO_CUDA_CORE,
          "tensor": _lib.GDR_ALGO_TENSOR, "tensor_split": _lib.GDR_ALGO_TENSOR_SPLIT}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _layer_io(gates, norm, q, v, g, beta):
    """The ``gdr_layer_io`` of a call's ``gates=(a, b, a_log, dt_bias)`` and
    ``norm=(z, weight, eps)``, the tensors it points at (kept alive by the
    caller), and the g / beta stand-ins for the shape contract."""
    io, keep = _lib.GdrLayerIO(), []
    if gates is not None:
        if g is not None or beta is not None:
            raise ValueError("with gates=(a, b, a_log, dt_bias), g and beta are None")
        a, b, a_log, dt_bias = gates
        if a.dtype not in _DTYPES or b.dtype != a.dtype:
            raise TypeError("the gate projections a, b share one dtype, f32, bf16 or f16")
        a, b = a.contiguous(), b.contiguous()
        a_log = a_log.to(torch.float32).contiguous()
        dt_bias = dt_bias.to(torch.float32).contiguous()
        keep += [a, b, a_log, dt_bias]
        io.gate_a, io.gate_b = a.data_ptr(), b.data_ptr()
        io.a_log, io.dt_bias = a_log.data_ptr(), dt_bias.data_ptr()
        io.gate_dtype = _DTYPES[a.dtype]
        g, beta = a, b  # for the shape contract only
    if norm is not None:
        z, weight, eps = norm
        if tuple(z.shape) != tuple(v.shape) or z.dtype != q.dtype:
            raise ValueError("the norm's gate z is shaped and typed like v and out")
        z = z.contiguous()
        weight = weight.to(torch.float32).contiguous()
        keep += [z, weight]
        io.norm_z, io.norm_weight, io.norm_eps = z.data_ptr(), weight.data_ptr(), float(eps)
    return io, keep, g, beta


@dataclasses.dataclass(frozen=True)
class GatedDeltaRule:
    """The rule's options (``delta_rule.rs:52-60``); the default is bunsen's
    ``Default``: ``qk_l2norm_eps = Some(1e-6)``, ``chunk_size = 64``."""

    qk_l2norm_eps: float | None = 1e-6
    chunk_size: int = 64
    algo: str = "auto"  # chunked calls: "auto", "cuda_core", "tensor" or "tensor_split"
    split_chunks: int = 0  # "tensor_split" / "auto": segment length in chunks, 0 = chosen

    def with_qk_l2norm_eps(self, eps: float | None) -> "GatedDeltaRule":
        return dataclasses.replace(self, qk_l2norm_eps=eps)

    def with_chunk_size(self, chunk_size: int) -> "GatedDeltaRule":
        return dataclasses.replace(self, chunk_size=chunk_size)

    # -- the two forms -------------------------------------------------------
    def recurrent(self, q, k, v, g, beta, state=None, *, cu_seqlens=None, out=None,
                  state_out=None, gates=None, norm=None):
        """One position at a time (``delta_rule.rs:182-209``). ``gates`` and
        ``norm`` run the layer's steps around the rule (see ``chunked``)."""
        return self._run("gdr_recurrent", q, k, v, g, beta, state, cu_seqlens, out, state_out,
                         gates, norm)

    def chunked(self, q, k, v, g, beta, state=None, *, cu_seqlens=None, out=None,
                state_out=None, gates=None, norm=None):
        """``chunk_size`` positions at a time (``delta_rule.rs:223-310``).

        ``gates=(a, b, a_log, dt_bias)``: g and beta (pass None for both) come
        from the layer's projections (``gated_delta_net.rs:422-426``).
        ``norm=(z, weight, eps)``: the output is the layer's gated RMS norm of
        the rule's output (``gated_delta_net.rs:439-440``)."""
        assert self.chunk_size > 0, "a chunk of at least one position"
        return self._run("gdr_chunked", q, k, v, g, beta, state, cu_seqlens, out, state_out,
                         gates, norm)

    def mixed(self, q, k, v, g, beta, state_pool, *, cu_seqlens, state_slots=None, out=None,
              workspace=None, gates=None, norm=None):
        """A continuous batch in one launch (``gdr_mixed``): the packed batch's
        length-1 sequences step as decode rows (``recurrent``), longer ones run
        as prefill segments (``chunked``). Sequence ``s`` updates its state in
        place at ``state_pool[state_slots[s]]``. Returns ``out``. ``gates`` and
        ``norm`` as for ``chunked`` (``gdr_mixed_layer``)."""
        assert self.chunk_size > 0, "a chunk of at least one position"
        io, keep = None, []
        if gates is not None or norm is not None:
            io, keep, g, beta = _layer_io(gates, norm, q, v, g, beta)
        check_shapes(q, k, v, g, beta, None, cu_seqlens)
        if q.dtype not in _DTYPES:
            raise TypeError(f"a continuous batch takes f32, bf16 or f16 q, k, v, not {q.dtype}")
        dev = q.device
        if dev.type != "cuda":
            raise RuntimeError("libgdr runs on CUDA tensors only")
        if state_pool.dtype != torch.float32 or not state_pool.is_contiguous():
            raise TypeError("the state pool is contiguous f32 [n_slots, H_v, d_k, d_v]")
        h_v, d_k, d_v = v.shape[-2], q.shape[-1], v.shape[-1]
        if tuple(state_pool.shape[1:]) != (h_v, d_k, d_v):
            raise ValueError(f"the state pool is [n_slots, {h_v}, {d_k}, {d_v}]")
        if gates is None:
            g = g.to(torch.float32).contiguous()
            beta = beta.to(torch.float32).contiguous()
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        cu_seqlens = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
        if state_slots is not None:
            state_slots = state_slots.to(device=dev, dtype=torch.int32).contiguous()
        if out is None:
            out = torch.empty(v.shape, dtype=q.dtype, device=dev)
        p = self.params(q, v, cu_seqlens)
        lib = _lib.load()
        need = lib.gdr_mixed_workspace_size(ctypes.byref(p))
        if workspace is None:
            workspace = torch.empty(max(need, 4), dtype=torch.uint8, device=dev)
        gp = None if gates is not None else g.data_ptr()
        bp = None if gates is not None else beta.data_ptr()
        if io is not None:
            status = lib.gdr_mixed_layer(
                ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), gp, bp,
                ctypes.byref(io), state_pool.data_ptr(), _ptr(state_slots), state_pool.shape[0],
                out.data_ptr(), cu_seqlens.data_ptr(), workspace.data_ptr(),
                workspace.numel() * workspace.element_size(), _stream(dev))
            _lib.check("gdr_mixed_layer", status)
            return out
        status = lib.gdr_mixed(
            ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), gp, bp,
            state_pool.data_ptr(), _ptr(state_slots), state_pool.shape[0],
            out.data_ptr(), cu_seqlens.data_ptr(), workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _stream(dev))
        _lib.check("gdr_mixed", status)
        return out

    def chunked_host(self, q, k, v, g, beta, state=None, *, cu_seqlens=None, out=None,
                     state_out=None, device=None, synchronize=True):
        """``chunked`` on host (CPU) tensors through ``gdr_chunked_host``: groups
        of sequences are copied to the GPU, run and copied back with copies in,
        kernels and copies out overlapping (pin the tensors for that). Runs on
        ``device`` (default: the current CUDA device) after the work already on
        its current stream; ``synchronize=False`` returns before the results
        have landed in ``out`` / ``state_out`` (wait on the stream first)."""
        assert self.chunk_size > 0, "a chunk of at least one position"
        packed = cu_seqlens is not None
        lead = 1 if packed else 2
        check_shapes(q, k, v, g, beta, state, cu_seqlens)
        if q.dtype not in _DTYPES:
            raise TypeError(f"q, k, v in f32, bf16 or f16, not {q.dtype}")
        if q.device.type != "cpu":
            raise RuntimeError("chunked_host takes host tensors; use chunked for CUDA tensors")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else \
            torch.device(device)
        if not synchronize:  # the copies read the caller's tensors after return
            ok = all(x.is_contiguous() for x in (q, k, v, g, beta)) and \
                g.dtype == beta.dtype == torch.float32 and \
                (state is None or (state.is_contiguous() and state.dtype == torch.float32))
            if not ok:
                raise ValueError("synchronize=False needs contiguous inputs, f32 g/beta/state")
        g = g.to(torch.float32).contiguous()
        beta = beta.to(torch.float32).contiguous()
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        n = (cu_seqlens.numel() - 1) if packed else q.shape[0]
        h_v, d_k, d_v = v.shape[-2], q.shape[-1], v.shape[-1]
        if out is None:
            out = torch.empty(v.shape[:lead] + (h_v, d_v), dtype=q.dtype).pin_memory()
        if state_out is None:
            state_out = torch.empty((n, h_v, d_k, d_v), dtype=torch.float32).pin_memory()
        if state is not None:
            state = state.to(torch.float32).contiguous()
        if packed:
            cu_seqlens = cu_seqlens.to(dtype=torch.int32).contiguous()
        p = self.params(q, v, cu_seqlens)
        with torch.cuda.device(dev):
            status = _lib.load().gdr_chunked_host(
                ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
                beta.data_ptr(), _ptr(state), out.data_ptr(), state_out.data_ptr(),
                _ptr(cu_seqlens), _stream(dev))
            _lib.check("gdr_chunked_host", status)
            if synchronize:
                torch.cuda.current_stream(dev).synchronize()
        return out, state_out

    def chunked_launches(self, q, v, cu_seqlens=None) -> int:
        """How many kernels ``chunked`` launches for these shapes (-1: the call
        would be rejected)."""
        p = self.params(q, v, cu_seqlens)
        return _lib.load().gdr_chunked_launches(ctypes.byref(p), int(cu_seqlens is not None))

    # -- plumbing ------------------------------------------------------------
    def params(self, q, v, cu_seqlens) -> _lib.GdrParams:
        if cu_seqlens is None:
            b, t, h_qk, d_k = q.shape
            n = b
        else:
            t, h_qk, d_k = q.shape
            b, n = 0, cu_seqlens.numel() - 1
        return _lib.GdrParams(
            batch=b, seq_len=t, n_seqs=n, heads_qk=h_qk, heads_v=v.shape[-2], d_k=d_k,
            d_v=v.shape[-1], chunk_size=self.chunk_size,
            use_l2norm=int(self.qk_l2norm_eps is not None),
            l2norm_eps=float(self.qk_l2norm_eps or 0.0),
            dtype=_lib.GDR_DTYPE_F64 if q.dtype == torch.float64 else _DTYPES[q.dtype],
            algo=_ALGOS[self.algo], split_chunks=self.split_chunks)

    def _run(self, fn, q, k, v, g, beta, state, cu_seqlens, out, state_out, gates=None,
             norm=None):
        if q.dtype == torch.float64:
            if gates is not None or norm is not None:
                raise TypeError("the layer's gates and norm take f32, bf16 or f16 tensors")
            return self._run_f64(fn + "_f64", q, k, v, g, beta, state, cu_seqlens, out,
                                 state_out)
        packed = cu_seqlens is not None
        lead = 1 if packed else 2
        io, keep = None, []
        if gates is not None or norm is not None:
            io, keep, g, beta = _layer_io(gates, norm, q, v, g, beta)
        check_shapes(q, k, v, g, beta, state, cu_seqlens)
        if q.dtype not in _DTYPES:
            raise TypeError(f"q, k, v in f32, bf16 or f16, not {q.dtype}")
        dev = q.device
        if dev.type != "cuda":
            raise RuntimeError("libgdr runs on CUDA tensors only")
        if gates is None:
            g = g.to(torch.float32).contiguous()
            beta = beta.to(torch.float32).contiguous()
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        n = (cu_seqlens.numel() - 1) if packed else q.shape[0]
        h_v, d_k, d_v = v.shape[-2], q.shape[-1], v.shape[-1]
        if out is None:
            out = torch.empty(v.shape[:lead] + (h_v, d_v), dtype=q.dtype, device=dev)
        if state_out is None:
            state_out = torch.empty((n, h_v, d_k, d_v), dtype=torch.float32, device=dev)
        if state is not None:
            state = state.to(torch.float32).contiguous()
        if packed:
            cu_seqlens = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
        p = self.params(q, v, cu_seqlens)
        if io is not None:
            status = getattr(_lib.load(), fn + "_layer")(
                ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                None if gates is not None else g.data_ptr(),
                None if gates is not None else beta.data_ptr(), ctypes.byref(io), _ptr(state),
                out.data_ptr(), state_out.data_ptr(), _ptr(cu_seqlens), _stream(dev))
            _lib.check(fn + "_layer", status)
            return out, state_out
        status = getattr(_lib.load(), fn)(
            ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
            beta.data_ptr(), _ptr(state), out.data_ptr(), state_out.data_ptr(),
            _ptr(cu_seqlens), _stream(dev))
        _lib.check(fn, status)
        return out, state_out


    def _run_f64(self, fn, q, k, v, g, beta, state, cu_seqlens, out, state_out):
        """f64 inputs: every tensor (g, beta, states, out) in f64."""
        packed = cu_seqlens is not None
        lead = 1 if packed else 2
        check_shapes(q, k, v, g, beta, state, cu_seqlens)
        dev = q.device
        if dev.type != "cuda":
            raise RuntimeError("libgdr runs on CUDA tensors only")
        f64 = torch.float64
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        g, beta = g.to(f64).contiguous(), beta.to(f64).contiguous()
        n = (cu_seqlens.numel() - 1) if packed else q.shape[0]
        h_v, d_k, d_v = v.shape[-2], q.shape[-1], v.shape[-1]
        if out is None:
            out = torch.empty(v.shape[:lead] + (h_v, d_v), dtype=f64, device=dev)
        if state_out is None:
            state_out = torch.empty((n, h_v, d_k, d_v), dtype=f64, device=dev)
        if out.dtype != f64 or state_out.dtype != f64:
            raise TypeError("an f64 call writes f64 outputs and states")
        if state is not None:
            state = state.to(f64).contiguous()
        if packed:
            cu_seqlens = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
        p = self.params(q, v, cu_seqlens)
        status = getattr(_lib.load(), fn)(
            ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
            beta.data_ptr(), _ptr(state), out.data_ptr(), state_out.data_ptr(),
            _ptr(cu_seqlens), _stream(dev))
        _lib.check(fn, status)
        return out, state_out


def check_shapes(q, k, v, g, beta, state, cu_seqlens) -> None:
    """bunsen's shape contracts (``delta_rule.rs:135-150``, ``:323-327``),
    dense ``[B, T, H, .]`` or packed ``[T_total, H, .]``."""
    packed = cu_seqlens is not None
    rank = 3 if packed else 4
    if q.dim() != rank:
        raise ValueError(f"q is {'[T, H, Dk]' if packed else '[B, T, H, Dk]'}; got {tuple(q.shape)}")
    if tuple(k.shape) != tuple(q.shape):
        raise ValueError(f"k {tuple(k.shape)} must match q {tuple(q.shape)}")
    lead = tuple(q.shape[: rank - 2])
    if v.dim() != rank or tuple(v.shape[: rank - 2]) != lead:
        raise ValueError(f"v {tuple(v.shape)} must share q's leading dims {lead}")
    h_qk, h_v = q.shape[-2], v.shape[-2]
    if h_v % h_qk != 0:
        raise ValueError(f"{h_qk} key heads must divide {h_v} value heads")
    for name, x in (("g", g), ("beta", beta)):
        if tuple(x.shape) != lead + (h_v,):
            raise ValueError(f"the rule's `{name}` is {'[T, H]' if packed else '[B, T, H]'}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("q, k and v share one dtype")
    if state is not None:
        n = (cu_seqlens.numel() - 1) if packed else q.shape[0]
        want = (n, h_v, q.shape[-1], v.shape[-1])
        if tuple(state.shape) != want:
            raise ValueError(f"the state is [B, H, Dk, Dv] = {want}; got {tuple(state.shape)}")
    if packed and (cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1):
        raise ValueError("cu_seqlens holds n_seqs + 1 offsets")
