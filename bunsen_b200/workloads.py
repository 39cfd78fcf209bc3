"""Seeded synthetic inputs of the rule's benchmark shapes.

Value distributions (all workloads): q, k ~ N(0, 1), then L2-normalised per
head vector; v ~ N(0, 1); beta = sigmoid(N(0, 1)); g = ln U(0.9, 0.999);
initial states, where a workload has them, N(0, 0.01) read as variance 0.01
(sigma 0.1). q/k/v are rounded to the workload's dtype once, and every consumer
(CUDA kernels, the CPU oracle) sees exactly those rounded values.

Workloads:
  fixture_f32   2 x 64 tokens, 4 heads, d 32, chunk 16, f32, zero state
  dense_prefill 8 x 4096 tokens, 16 q/k heads, 32 v heads, d 128, chunk 64,
                bf16, zero state
  ragged_prefill 131072 tokens in 64 sequences, lengths lognormal(7, 1)
                clipped to [16, 16384] and rescaled to the total; heads and
                dims as dense_prefill; initial states
  decode        256 rows x 1 token, heads and dims as dense_prefill, states
  mixed         8 prefill segments x 2048 tokens + 1024 decode rows, every
                sequence continuing from a state

``scale`` shrinks a workload (fewer sequences / rows / tokens) for tests that
compare against the CPU oracle.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import torch


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    seqlens: tuple[int, ...]   # tokens per sequence (1 = a decode row)
    heads_qk: int
    heads_v: int
    d_k: int
    d_v: int
    chunk: int
    dtype: torch.dtype
    with_state: bool
    packed: bool               # cu_seqlens (ragged) rather than dense [B, T]

    @property
    def tokens(self) -> int:
        return int(sum(self.seqlens))

    @property
    def n_seqs(self) -> int:
        return len(self.seqlens)


def ragged_lengths(total: int = 131072, n: int = 64, mu: float = 7.0, sigma: float = 1.0,
                   lo: int = 16, hi: int = 16384, seed: int = 2024) -> list[int]:
    """Lognormal lengths clipped to [lo, hi], rescaled to sum to `total`,
    rounded, re-clipped; the residual goes to the longest."""
    rng = np.random.default_rng(seed)
    x = np.clip(rng.lognormal(mu, sigma, n), lo, hi)
    x = np.clip(np.rint(x * total / x.sum()), lo, hi).astype(np.int64)
    x[np.argmax(x)] += total - int(x.sum())
    assert x.sum() == total and x.min() >= 1
    return [int(v) for v in x]


def get(name: str, scale: float = 1.0) -> Workload:
    """A named workload; `scale` < 1 keeps its shapes per sequence but fewer
    sequences (and, for the ragged pack, proportionally shorter ones)."""
    def n(x: int) -> int:
        return max(1, int(round(x * scale)))

    if name == "fixture_f32":
        return Workload(name, (64,) * 2, 4, 4, 32, 32, 16, torch.float32, False, False)
    if name == "dense_prefill":
        return Workload(name, (4096,) * n(8), 16, 32, 128, 128, 64, torch.bfloat16, False, False)
    if name == "ragged_prefill":
        lens = ragged_lengths(total=n(131072), n=n(64), hi=max(16, n(16384)))
        return Workload(name, tuple(lens), 16, 32, 128, 128, 64, torch.bfloat16, True, True)
    if name == "decode":
        return Workload(name, (1,) * n(256), 16, 32, 128, 128, 64, torch.bfloat16, True, False)
    if name == "mixed":
        return Workload(name, (2048,) * n(8) + (1,) * n(1024), 16, 32, 128, 128, 64,
                        torch.bfloat16, True, True)
    raise KeyError(name)


def make_inputs(w: Workload, device: str | torch.device = "cpu", seed: int = 1234) -> dict:
    """q, k, v, g, beta (+ state, cu_seqlens) for `w`, generated on `device`
    with a seeded torch generator. Dense workloads are [B, T, H, .]; packed
    ones [T_total, H, .] with cu_seqlens."""
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    t = w.tokens
    f32 = dict(device=device, dtype=torch.float32)

    def normal(*shape):
        return torch.randn(*shape, generator=gen, **f32)

    def unit(x):
        return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12)

    q = unit(normal(t, w.heads_qk, w.d_k)).to(w.dtype)
    k = unit(normal(t, w.heads_qk, w.d_k)).to(w.dtype)
    v = normal(t, w.heads_v, w.d_v).to(w.dtype)
    beta = torch.sigmoid(normal(t, w.heads_v))
    g = torch.log(torch.rand(t, w.heads_v, generator=gen, **f32) * (0.999 - 0.9) + 0.9)
    out = {"q": q, "k": k, "v": v, "g": g, "beta": beta}
    if w.with_state:
        out["state"] = normal(w.n_seqs, w.heads_v, w.d_k, w.d_v) * 0.1
    if w.packed:
        cu = np.concatenate([[0], np.cumsum(w.seqlens)]).astype(np.int32)
        out["cu_seqlens"] = torch.from_numpy(cu).to(device)
    else:
        b, tt = w.n_seqs, w.seqlens[0]
        for key in ("q", "k", "v", "g", "beta"):
            out[key] = out[key].reshape((b, tt) + out[key].shape[1:])
    return out


def to_numpy_f32(x: torch.Tensor) -> np.ndarray:
    """The f32 values a tensor holds (bf16 widened exactly), on the host."""
    return x.detach().to("cpu", torch.float32).numpy()
