"""Runs one kernel family on one named workload a few times: the small, fixed
cases the committed ncu summaries under profiles/ are captured on.

    python -m bunsen_b200.profile_case ragged_prefill --scale 0.25 --iters 3
    python -m bunsen_b200.profile_case decode --iters 3
    python -m bunsen_b200.profile_case ragged_prefill --shard 8 --algo tensor_split
    python -m bunsen_b200.profile_case conv --scale 0.25         # the layer's conv
    python -m bunsen_b200.profile_case layer_prefill --scale 0.25  # gates + norm fused
    python -m bunsen_b200.profile_case dense_prefill --dtype f32  # the f32 chunked kernel

Prints the mean CUDA-event time per call. `--shard N` keeps the heads one GPU
of an N-way head shard holds (H_qk / N key heads with their value heads).

Workloads and value distributions are those of bunsen_b200.workloads (inputs
larger than L2 at the scales used); `conv` and `layer_prefill` take the ragged
pack's shapes.
"""

from __future__ import annotations

import argparse

import torch

from . import workloads
from .layer import causal_conv1d
from .rule import GatedDeltaRule


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", choices=["ragged_prefill", "dense_prefill", "decode", "mixed",
                                         "conv", "layer_prefill"])
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--algo", default="auto",
                    choices=["auto", "tensor", "tensor_split", "cuda_core"])
    ap.add_argument("--split-chunks", type=int, default=0)
    ap.add_argument("--shard", type=int, default=1)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16", "f32"],
                    help="dtype of q, k, v and out (the workloads are bf16)")
    args = ap.parse_args()
    base = {"conv": "ragged_prefill", "layer_prefill": "ragged_prefill"}.get(args.workload,
                                                                             args.workload)
    w = workloads.get(base, scale=args.scale)
    x = workloads.make_inputs(w, "cuda", seed=1)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[args.dtype]
    x = {k: (v.to(dt) if k in ("q", "k", "v") else v) for k, v in x.items()}
    if args.shard > 1:
        hq, hv = w.heads_qk // args.shard, w.heads_v // args.shard
        heads = {"q": hq, "k": hq, "v": hv, "g": hv, "beta": hv}
        lead = 1 if w.packed else 2
        x = {k: (v[(slice(None),) * lead + (slice(0, heads[k]),)].contiguous() if k in heads
                 else v[:, :hv].contiguous() if k == "state" else v) for k, v in x.items()}
    rule = GatedDeltaRule(chunk_size=w.chunk, algo=args.algo, split_chunks=args.split_chunks)
    hv = x["v"].shape[-2]
    gen = torch.Generator(device="cuda").manual_seed(2)
    if args.workload == "conv":  # the layer's conv of this pack: 2 H_qk d_k + H_v d_v channels
        hq = x["q"].shape[-2]
        c = 2 * hq * w.d_k + hv * w.d_v
        xc = torch.randn(w.tokens, c, device="cuda", generator=gen).bfloat16()
        wc = torch.randn(c, 4, device="cuda", generator=gen).bfloat16()
        st = torch.randn(w.n_seqs, 3, c, device="cuda", generator=gen)
        run = lambda: causal_conv1d(xc, wc, st, cu_seqlens=x["cu_seqlens"], silu=True,  # noqa
                                    splits=(hq * w.d_k, 2 * hq * w.d_k))
    elif args.workload == "layer_prefill":  # the prefill with the layer's gates and norm
        a = torch.randn(w.tokens, hv, device="cuda", generator=gen).bfloat16()
        b = torch.randn(w.tokens, hv, device="cuda", generator=gen).bfloat16()
        a_log = torch.log(torch.rand(hv, device="cuda", generator=gen) * 0.2 + 0.01)
        dt_bias = torch.randn(hv, device="cuda", generator=gen) * 0.1
        z = torch.randn(w.tokens, hv, w.d_v, device="cuda", generator=gen).bfloat16()
        nw = torch.rand(w.d_v, device="cuda", generator=gen) + 0.5
        run = lambda: rule.chunked(x["q"], x["k"], x["v"], None, None, x["state"],  # noqa
                                   cu_seqlens=x["cu_seqlens"], gates=(a, b, a_log, dt_bias),
                                   norm=(z, nw, 1e-6))
    elif args.workload == "decode":
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
    print(f"{args.workload} scale {args.scale} shard {args.shard} {args.algo} {args.dtype}: "
          f"{e0.elapsed_time(e1) / args.iters:.4f} ms per call, "
          f"{w.tokens} tokens, {w.n_seqs} sequences")


if __name__ == "__main__":
    main()
