"""Head sharding across the GPUs of one box.

Heads are independent in the rule: value head h touches only its own state
and its key head h // (H_v / H_qk) (the `repeat_interleave` mapping of
``gated_delta_net.rs:404-419``). So P ranks split the key-head groups: rank r
owns key heads [r H_qk / P, (r + 1) H_qk / P) and the value heads that read
them; every rank sees the whole token axis (and ``cu_seqlens``) and runs the
same kernels on its slice. The hot path has no collective. Outputs can be
gathered across ranks (``gather_heads``) to check a sharded run against a
single-GPU one.
"""

from __future__ import annotations

import dataclasses

import torch


@dataclasses.dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    heads_qk: int
    heads_v: int

    def __post_init__(self):
        if self.heads_qk % self.world:
            raise ValueError(f"{self.world} ranks must divide the {self.heads_qk} key heads")
        if self.heads_v % self.heads_qk:
            raise ValueError(f"{self.heads_qk} key heads must divide {self.heads_v} value heads")

    @property
    def qk(self) -> slice:
        n = self.heads_qk // self.world
        return slice(self.rank * n, (self.rank + 1) * n)

    @property
    def v(self) -> slice:
        g = self.heads_v // self.heads_qk
        return slice(self.qk.start * g, self.qk.stop * g)

    def take(self, inputs: dict) -> dict:
        """This rank's slice of the rule's inputs (dense [B, T, H, .] or packed
        [T, H, .] token tensors; states [N, H_v, d_k, d_v]), contiguous."""
        out = {}
        for name, t in inputs.items():
            if name in ("q", "k"):
                out[name] = t[..., self.qk, :].contiguous()
            elif name == "v":
                out[name] = t[..., self.v, :].contiguous()
            elif name in ("g", "beta"):
                out[name] = t[..., self.v].contiguous()
            elif name == "state":
                out[name] = t[:, self.v].contiguous()
            else:
                out[name] = t
        return out


def gather_heads(local: torch.Tensor, shard: HeadShard, head_dim: int, group=None):
    """All ranks' slices of a head-sharded tensor, concatenated back along
    the head axis `head_dim` (all_gather over the process group: NCCL between
    GPUs, gloo on the host). Verification only: not on the hot path."""
    import torch.distributed as dist

    parts = [torch.empty_like(local) for _ in range(shard.world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=head_dim)


def max_over_ranks(ms: float, device=None, group=None) -> float:
    """The slowest rank's time: a sharded step ends when its last rank does."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return ms
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
