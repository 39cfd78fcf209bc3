"""Head sharding on CPU ranks (gloo, world size 2): each rank runs its key-head
group's slice, the gathered result is the unsharded run exactly (heads are
independent), and the step time is the slowest rank's."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bunsen_b200.sharding import HeadShard, gather_heads, max_over_ranks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed=0, t=40, hq=4, hv=8, d=8):
    g = torch.Generator().manual_seed(seed)
    lens = [17, 1, 22]
    return {"q": torch.randn(t, hq, d, generator=g), "k": torch.randn(t, hq, d, generator=g),
            "v": torch.randn(t, hv, d, generator=g),
            "g": -torch.rand(t, hv, generator=g), "beta": torch.rand(t, hv, generator=g),
            "state": torch.randn(len(lens), hv, d, d, generator=g),
            "cu_seqlens": torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)}


def _run(x):
    from oracle import oracle

    n = lambda t: t.numpy()  # noqa: E731
    o, s = oracle.chunked(n(x["q"]), n(x["k"]), n(x["v"]), n(x["g"]), n(x["beta"]),
                          n(x["state"]), cu_seqlens=n(x["cu_seqlens"]), chunk_size=8, threads=1)
    return torch.from_numpy(o), torch.from_numpy(s)


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = _inputs()
        sh = HeadShard(rank, world, heads_qk=4, heads_v=8)
        o, s = _run(sh.take(x))
        o_all = gather_heads(o, sh, head_dim=1)
        s_all = gather_heads(s, sh, head_dim=1)
        slowest = max_over_ranks(10.0 + rank)
        if rank == 0:
            wo, ws = _run(x)
            results.put((torch.equal(o_all, wo), torch.equal(s_all, ws), slowest))
    finally:
        dist.destroy_process_group()


def test_two_rank_head_sharding_equals_one_pass():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    same_out, same_state, slowest = results.get(timeout=5)
    assert same_out and same_state
    assert slowest == 11.0


def test_shard_slices_follow_repeat_interleave():
    sh = HeadShard(1, 4, heads_qk=16, heads_v=32)
    assert (sh.qk.start, sh.qk.stop) == (4, 8)
    assert (sh.v.start, sh.v.stop) == (8, 16)  # value heads reading key heads 4..7
    with pytest.raises(ValueError):
        HeadShard(0, 3, heads_qk=16, heads_v=32)
    with pytest.raises(ValueError):
        HeadShard(0, 2, heads_qk=4, heads_v=6)
