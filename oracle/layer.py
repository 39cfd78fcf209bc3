"""numpy restatements of the gated DeltaNet layer's steps around the rule --
TEST INFRASTRUCTURE ONLY (the tests and the benchmark's CPU legs use it; the
product never imports it).

Each function follows bunsen's own code, in f32 unless stated:

* ``causal_conv1d``: ``causal_depthwise_conv1d``
  (``crates/public/bunsen/src/ops/transformers/linear_attention/causal_conv.rs:36-69``):
  ``y[t, c] = sum_j w[c, j] x[t - (K - 1) + j, c]``, the inputs before a
  sequence's first position from its state (zeros without one), the sum taken
  in tap order; the next state is the last ``K - 1`` inputs of the window
  ``[state, x]``. The layer then applies silu (``gated_delta_net.rs:401``) and
  splits the channels into q, k, v (``:404-420``).
* ``gates``: ``gated_delta_net.rs:422-426``: ``g = -exp(A_log) *
  softplus(a + dt_bias)`` in f32 (``Widening::F32`` over ``a``, ``A_log`` and
  ``dt_bias``); ``beta = sigmoid(b)`` on the projection's own tensor, so the
  value keeps the projection's dtype: rounded to bf16 for a bf16 model
  (``beta_dtype="bf16"``), before the rule widens it back to f32.
* ``gated_norm``: ``gated_delta_net.rs:439-440`` through ``GatedNorm``
  (``blocks/norm/gated_norm.rs``) and ``Gate::forward``
  (``burner/module/gate.rs:89-102``): an RMS norm over the last axis with its
  weight, times ``silu(z)`` computed in f32.
* ``reorder``: ``DeltaNetState::reorder`` (``linear_attention/state.rs:112-135``):
  row ``r`` of the result is row ``sources[r]``.
"""

from __future__ import annotations

import numpy as np


def _spans(n_tokens: int, cu_seqlens, batch: int | None):
    if cu_seqlens is None:
        t = n_tokens // batch
        return [(s * t, (s + 1) * t) for s in range(batch)]
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    return [(int(cu[s]), int(cu[s + 1])) for s in range(len(cu) - 1)]


def silu(x):
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1) + np.exp(-x))).astype(np.float32)


def causal_conv1d(x, weight, state=None, *, cu_seqlens=None, activation=False):
    """x ``[T, C]`` packed (with ``cu_seqlens``; one sequence without) or
    ``[B, T, C]``; weight ``[C, K]`` (oldest tap first); state
    ``[N, K - 1, C]`` or None. Returns ``(y, next_state)``: y with x's shape
    (silu applied when ``activation``), next_state ``[N, K - 1, C]`` f32."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(weight, dtype=np.float32)
    flat = x.reshape(-1, x.shape[-1])
    c, k = w.shape
    if cu_seqlens is None and x.ndim == 2:
        cu_seqlens = [0, flat.shape[0]]
    spans = _spans(flat.shape[0], cu_seqlens, x.shape[0] if cu_seqlens is None else None)
    y = np.zeros_like(flat)
    nxt = np.zeros((len(spans), k - 1, c), dtype=np.float32)
    for s, (a, b) in enumerate(spans):
        prev = (np.zeros((k - 1, c), np.float32) if state is None
                else np.asarray(state[s], dtype=np.float32))
        padded = np.concatenate([prev, flat[a:b]], axis=0)  # [K - 1 + L, C]
        length = b - a
        acc = padded[0:length] * w[:, 0]
        for j in range(1, k):
            acc = acc + padded[j:j + length] * w[:, j]
        y[a:b] = acc
        nxt[s] = padded[length:]
    if activation:
        y = silu(y)
    return y.reshape(x.shape), nxt


def round_bf16(x):
    """f32 values rounded to the nearest bf16 (ties to even), as f32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def gates(a, b, a_log, dt_bias, beta_dtype=None):
    """``(g, beta)`` from the projections ``a, b [..., H]`` and the per-head
    ``A_log, dt_bias [H]``; ``beta_dtype="bf16"``: the projections are bf16
    tensors, and beta is rounded to bf16."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    sp = np.logaddexp(np.float32(0), a + np.asarray(dt_bias, np.float32)).astype(np.float32)
    g = (-np.exp(np.asarray(a_log, np.float32)) * sp).astype(np.float32)
    beta = (np.float32(1) / (np.float32(1) + np.exp(-b))).astype(np.float32)
    if beta_dtype == "bf16":
        beta = round_bf16(beta)
    elif beta_dtype is not None:
        raise ValueError(f"beta_dtype is None (f32) or 'bf16', not {beta_dtype!r}")
    return g, beta


def gated_norm(x, z, weight, eps):
    """``rmsnorm(x) * weight * silu(z)`` over the last axis."""
    x = np.asarray(x, dtype=np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True)
    y = x / np.sqrt(var + np.float32(eps))
    return (y * np.asarray(weight, np.float32) * silu(z)).astype(np.float32)


def reorder(pool, sources):
    """Row ``r`` of the result is row ``sources[r]`` of ``pool``."""
    pool = np.asarray(pool)
    return pool[np.asarray(sources, dtype=np.int64)].copy()
