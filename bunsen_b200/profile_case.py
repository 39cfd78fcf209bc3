"""Runs one kernel family on one named workload a few times: the small, fixed
cases the committed ncu summaries under profiles/ are captured on.

    python -m bunsen_b200.profile_case ragged_prefill --scale 0.25 --iters 3
    python -m bunsen_b200.profile_case decode --iters 3
    python -m bunsen_b200.profile_case ragged_prefill --shard 8 --algo tensor_split

Prints the mean CUDA-event time per call. `--shard N` keeps the heads one GPU
of an N-way head shard holds (H_qk / N key heads with their value heads).

Workloads and value distributions
are those of bunsen_b200.workloads (inputs larger than L2 at the scales used).
"""

from __future__ import annotations

import argparse

import torch

from . import workloads
from .rule import GatedDeltaRule


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", choices=["ragged_prefill", "dense_prefill", "decode", "mixed"])
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--algo", default="auto",
                    choices=["auto", "tensor", "tensor_split", "cuda_core"])
    ap.add_argument("--split-chunks", type=int, default=0)
    ap.add_argument("--shard", type=int, default=1)
    args = ap.parse_args()
    w = workloads.get(args.workload, scale=args.scale)
    x = workloads.make_inputs(w, "cuda", seed=1)
    if args.shard > 1:
        hq, hv = w.heads_qk // args.shard, w.heads_v // args.shard
        heads = {"q": hq, "k": hq, "v": hv, "g": hv, "beta": hv}
        lead = 1 if w.packed else 2
        x = {k: (v[(slice(None),) * lead + (slice(0, heads[k]),)].contiguous() if k in heads
                 else v[:, :hv].contiguous() if k == "state" else v) for k, v in x.items()}
    rule = GatedDeltaRule(chunk_size=w.chunk, algo=args.algo, split_chunks=args.split_chunks)
    if args.workload == "decode":
        st = x["state"]
        run = lambda: rule.recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], st,  # noqa
                                     state_out=st)
    elif args.workload == "mixed":
        pool = x["state"]
        run = lambda: rule.mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], pool,  # noqa
                                 cu_seqlens=x["cu_seqlens"])
    else:
        run = lambda: rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"],  # noqa
                                   x.get("state"), cu_seqlens=x.get("cu_seqlens"))
    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.iters):
        run()
    e1.record()
    e1.synchronize()
    print(f"{args.workload} scale {args.scale} shard {args.shard} {args.algo}: "
          f"{e0.elapsed_time(e1) / args.iters:.4f} ms per call, "
          f"{w.tokens} tokens, {w.n_seqs} sequences")


if __name__ == "__main__":
    main()
