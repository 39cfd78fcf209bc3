#!/usr/bin/env python3
"""Benchmark of the gated delta rule on B200s.

One JSON line (rank 0). The headline `value` is ragged prefill tokens/s: one
step is one gdr_chunked call over the whole ragged pack (131072 tokens in 64
lognormal sequences, 16 q/k heads, 32 v heads, d 128, chunk 64, bf16, f32
initial states), inputs resident in HBM (2.3 GB, larger than L2, so no flush
is needed). Sub-objects carry the other workloads at the same N:
  dense    8 x 4096 tokens, zero initial state (gdr_chunked)
  dense_f32  the same with f32 q, k, v (the register-tiled f32 CUDA-core kernel)
  decode   64 consecutive single-token steps over 256 rows, f32 states
           [256, 32, 128, 128] updated in place (gdr_recurrent)
  mixed    8 prefill segments x 2048 tokens + 1024 decode rows in one
           gdr_mixed launch, states in place in a slot pool
With N GPUs (torchrun), the key-head groups are sharded (rank r: key heads
[16r/N, 16(r+1)/N) and their value heads) over the same tokens; no data
crosses GPUs on the hot path; every time is the maximum over ranks; `value`
counts the pack's tokens (all heads) once -- strong scaling. `--verify`
gathers the sharded outputs (NCCL all_gather, outside the timed region) and
compares them with an unsharded run on rank 0.

`cpu_baseline` (rank 0, one GPU) and `--impl reference` time the CPU oracle --
a C++ restatement of bunsen's burn rule (the reference itself is Rust and
cannot be built here), OpenMP over (sequence, head) pairs on every host core
the process may use -- on the whole of each workload: the ragged pack (the
reference arm's step), the dense batch, one decode step and the mixed batch.

`roofline` is the attainable roof of one call, max(FLOPs / bf16 tensor peak,
bytes / HBM bandwidth), with the burst tensor peak (timed regions here last
tens of milliseconds) and the measured peaks of MEASURED_PEAKS.json.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from bunsen_b200 import _lib, workloads  # noqa: E402
from bunsen_b200.rule import GatedDeltaRule  # noqa: E402
from bunsen_b200.sharding import HeadShard  # noqa: E402

METRIC = "GDR prefill tokens/sec (ragged) and decode state-update GB/s vs HBM peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# -- roofline bookkeeping --------------------------------------------------------
def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def prefill_flops(w: workloads.Workload, heads_v: int) -> float:
    """Algorithmic FLOPs: per token per value head 10 C d + 6 d^2 + (2/3) C^2
    (a chunk's five C x C x d and three C x d x d matmuls, and the C^3/3 of the
    inverse)."""
    c, d = w.chunk, w.d_k
    return (10 * c * d + 6 * d * d + (2.0 / 3.0) * c * c) * w.tokens * heads_v


def prefill_bytes(w: workloads.Workload, heads_qk: int, heads_v: int) -> float:
    """Algorithmic HBM bytes: q, k once per key head, v and out in bf16, g and
    beta in f32; states written, and read when the workload has them."""
    per_tok = heads_qk * w.d_k * 2 * 2 + heads_v * w.d_v * 2 * 2 + heads_v * 4 * 2
    states = w.n_seqs * heads_v * w.d_k * w.d_v * 4 * (2 if w.with_state else 1)
    return float(w.tokens * per_tok + states)


def measured_traffic(tokens_heads: float) -> float | None:
    """DRAM bytes of one prefill call over `tokens_heads` token-heads, scaled
    from the ncu capture recorded in profiles/traffic.json (every launch of
    one call of the default path, summed)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    rec = json.loads(p.read_text()).get("ragged_prefill_call")
    if not rec:
        return None
    return rec["dram_bytes"] / rec["token_heads"] * tokens_heads


def roofline(flops: float, nbytes: float, kern_ms: float, pk: dict, pk_kind: str,
             traffic: float | None, tensor_peak: str = "burst") -> dict:
    """The attainable roof of one call, t_min = max(FLOPs / tensor peak, bytes /
    HBM bandwidth), names the binding roof (`bound`); `frac` = t_min / the
    measured time, which is the achieved rate over that roof's peak. The
    tensor peak is the burst figure for calls timed in a region well under a
    second, the sustained one for long regions."""
    tc = pk["bf16_tflops"] if tensor_peak == "burst" else pk["bf16_tflops_sustained"]
    t_flop = flops / (tc * 1e12)
    t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
    s = kern_ms * 1e-3
    if t_flop >= t_hbm:
        out = {"bound": "tensor", "achieved": flops / s / 1e12, "peak": tc, "unit": "TFLOP/s"}
    else:
        out = {"bound": "hbm", "achieved": nbytes / s / 1e9, "peak": pk["hbm_gbs"],
               "unit": "GB/s"}
    out["frac"] = out["achieved"] / out["peak"]
    out.update(traffic=traffic, peak_source=f"{pk_kind} ({tensor_peak} tensor peak)",
               attainable_ms=1e3 * max(t_flop, t_hbm), measured_ms=kern_ms,
               flops_per_launch=flops, bytes_per_launch=nbytes,
               tflops=flops / s / 1e12, gbs=nbytes / s / 1e9,
               tensor_frac=flops / s / 1e12 / tc, hbm_frac=nbytes / s / 1e9 / pk["hbm_gbs"])
    return out


# -- clocks, ranks, timing ---------------------------------------------------------
class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows: list[list[str]] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        num = lambda x: float(x) if x.replace(".", "").isdigit() else None  # noqa: E731
        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
        return self

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if self.pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def timed(step, k: int, w: int, dist: Dist, stream) -> tuple[float, list[float]]:
    """W warm-up steps, then K timed steps bracketed by a barrier and a device
    synchronize on both sides; CUDA events on the launching stream around each
    step. Returns (max-over-ranks total ms, this rank's per-step ms)."""
    for _ in range(w):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(k + 1)]
    evs[0].record(stream)
    for i in range(k):
        step()
        evs[i + 1].record(stream)
    evs[-1].synchronize()
    torch.cuda.synchronize()
    dist.barrier()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(k)]
    return dist.max(evs[0].elapsed_time(evs[-1])), per


# -- the CPU baseline ------------------------------------------------------------
# The oracle (a C++ restatement of bunsen's burn rule, OpenMP over (sequence,
# head) pairs) on the host's cores, on the same workloads as the GPU legs.
def cpu_threads() -> int:
    """Every core this process may run on: a launcher's OMP_NUM_THREADS
    (torchrun sets 1 per rank) is not the host's thread budget for the one
    CPU run."""
    from oracle import oracle

    return (len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity")
            else oracle.max_threads())


def cpu_inputs(name: str, seed: int = 99) -> tuple[workloads.Workload, dict]:
    """A workload's inputs as f32 numpy arrays on the host (bf16 values
    widened exactly, as bunsen widens them)."""
    w = workloads.get(name)
    x = workloads.make_inputs(w, "cpu", seed=seed)
    f = {k: workloads.to_numpy_f32(v) for k, v in x.items() if k != "cu_seqlens"}
    if "cu_seqlens" in x:
        f["cu_seqlens"] = x["cu_seqlens"].numpy().astype(np.int32)
    return w, f


def cpu_runner(name: str, threads: int):
    """(workload, one run of the whole workload on the oracle, what it is)."""
    from oracle import oracle

    w, f = cpu_inputs(name)
    args = lambda sl=slice(None): [f[k][sl] for k in ("q", "k", "v", "g", "beta")]  # noqa: E731
    # Output buffers made once and reused by every run (as an allocator reuses
    # them), so the runs time the rule, not first-touch page faults.
    t, n = w.tokens, w.n_seqs
    out = np.empty((t, w.heads_v, w.d_v), np.float32)
    st = np.empty((n, w.heads_v, w.d_k, w.d_v), np.float32)
    if name in ("ragged_prefill", "dense_prefill"):
        def run():
            oracle.chunked(*args(), f.get("state"), cu_seqlens=f.get("cu_seqlens"),
                           chunk_size=w.chunk, threads=threads, out=out, state_out=st)
        what = "f32 chunked oracle"
    elif name == "decode":
        def run():
            oracle.recurrent(*args(), f["state"], threads=threads, out=out, state_out=st)
        what = "f32 recurrent oracle, one step"
    elif name == "mixed":
        n_pre = sum(1 for L in w.seqlens if L > 1)
        t_pre = sum(L for L in w.seqlens if L > 1)
        cu = f["cu_seqlens"][:n_pre + 1]
        pre, dec = args(slice(0, t_pre)), [a[:, None] for a in args(slice(t_pre, None))]

        def run():
            oracle.chunked(*pre, f["state"][:n_pre], cu_seqlens=cu, chunk_size=w.chunk,
                           threads=threads, out=out[:t_pre], state_out=st[:n_pre])
            oracle.recurrent(*dec, f["state"][n_pre:], threads=threads, out=out[t_pre:],
                             state_out=st[n_pre:])
        what = "f32 chunked oracle on the prefill segments + recurrent on the decode rows"
    else:
        raise KeyError(name)
    return w, run, f"the whole {name} workload ({what}, {threads} threads, outputs reused)"


def time_cpu(run, seconds: float) -> tuple[float, int]:
    """Mean seconds per run: at least one run, more until `seconds` pass."""
    t0 = time.perf_counter()
    reps = 0
    while reps < 1 or (time.perf_counter() - t0 < seconds and reps < 100):
        run()
        reps += 1
    return (time.perf_counter() - t0) / reps, reps


def cpu_baselines(seconds: float = 5.0) -> dict:
    """The oracle on every workload of the GPU legs, in the GPU legs' units."""
    threads = cpu_threads()
    res = {}
    for name in ("ragged_prefill", "dense_prefill", "decode", "mixed"):
        w, run, desc = cpu_runner(name, threads)
        dt, reps = time_cpu(run, seconds)
        base = {"cores": threads, "kind": "port", "sample": f"{desc}; {reps} runs"}
        if name == "decode":
            state_rw = 2.0 * w.n_seqs * w.heads_v * w.d_k * w.d_v * 4
            res[name] = {"value": state_rw / dt / 1e9, "unit": "GB/s", **base}
        elif name == "mixed":
            res[name] = {"value": 1e3 * dt, "unit": "ms", "higher_is_better": False, **base}
        else:
            res[name] = {"value": w.tokens / dt, "unit": "tokens/s", **base}
        del run
    return res


def headline_config(w: workloads.Workload, world: int) -> dict:
    """The `config` of the headline line, the same in both arms."""
    return {"workload": "ragged_prefill", "tokens": w.tokens, "n_seqs": w.n_seqs,
            "max_len": max(w.seqlens), "heads_qk": w.heads_qk, "heads_v": w.heads_v,
            "d": w.d_k, "chunk": w.chunk, "parallelism": f"heads{world}",
            "l2": "inputs larger than L2 (no flush)"}


def run_reference(args, dist: Dist) -> None:
    """The reference arm: the oracle's chunked form over the whole ragged
    workload on all the host's cores, one run per step, on rank 0 only."""
    if dist.rank != 0:
        return
    threads = cpu_threads()
    w, run, desc = cpu_runner("ragged_prefill", threads)
    for _ in range(args.warmup):
        run()
    per = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        per.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(per)
    tok_s = w.tokens / (ms * 1e-3)
    line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": headline_config(w, args.gpus),
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads,
                             "kind": "port", "sample": desc},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# -- the GPU arm --------------------------------------------------------------------
def shard_of(w: workloads.Workload, dist: Dist) -> HeadShard:
    return HeadShard(dist.rank, dist.world, w.heads_qk, w.heads_v)


def bench_prefill(name: str, args, dist, dev, stream, pk, pk_kind, e2e=False, verify=False):
    w = workloads.get(name)
    sh = shard_of(w, dist)
    full = workloads.make_inputs(w, dev, seed=1234)
    x = sh.take(full)
    hq, hv = sh.qk.stop - sh.qk.start, sh.v.stop - sh.v.start
    rule = GatedDeltaRule(chunk_size=w.chunk)
    lead = x["v"].shape[:-2]
    out = torch.empty(lead + (hv, w.d_v), dtype=w.dtype, device=dev)
    st_out = torch.empty(w.n_seqs, hv, w.d_k, w.d_v, dtype=torch.float32, device=dev)

    def step():
        rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x.get("state"),
                     cu_seqlens=x.get("cu_seqlens"), out=out, state_out=st_out)

    with Clocks(dist.local) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, dist, stream)
    ms = total_ms / args.steps
    launches = rule.chunked_launches(x["q"], x["v"], x.get("cu_seqlens"))
    res = {"tokens": w.tokens, "ms_per_step": ms, "value": w.tokens / (ms * 1e-3),
           "unit": "tokens/s", "clocks": clk.summary(), "gpu_launches": args.steps * launches,
           "roofline": roofline(prefill_flops(w, hv), prefill_bytes(w, hq, hv),
                                statistics.mean(per), pk, pk_kind,
                                measured_traffic(w.tokens * hv))}
    if verify and dist.world > 1:
        from bunsen_b200.sharding import gather_heads

        step()
        o_all = gather_heads(out, sh, head_dim=out.dim() - 2)
        s_all = gather_heads(st_out, sh, head_dim=1)
        if dist.rank == 0:
            o1, s1 = rule.chunked(full["q"], full["k"], full["v"], full["g"], full["beta"],
                                  full.get("state"), cu_seqlens=full.get("cu_seqlens"))
            # Per GPU the call may cut long sequences into segments (fewer
            # heads, fewer CTAs to fill), so the check is the bf16 tolerance.
            eo = ((o_all.float() - o1.float()).abs().max() / o1.float().abs().max()).item()
            es = ((s_all - s1).abs().max() / s1.abs().max()).item()
            res["verified"] = bool(eo <= 2e-2 and es <= 1e-2)
            res["verify_rel_err"] = {"out": eo, "state": es}
    del full
    if e2e:
        res["e2e"] = bench_e2e(w, x, rule, out, st_out, args, dist, dev, stream)
    return res


def bench_dense_f32(args, dist, dev, stream, pk, pk_kind) -> dict:
    """The dense configuration with f32 q, k, v (bunsen's f32 models): the
    register-tiled f32 CUDA-core chunked kernel, every product an f32 FMA."""
    w = workloads.get("dense_prefill")
    sh = shard_of(w, dist)
    x = sh.take(workloads.make_inputs(w, dev, seed=1234))
    x = {k: (v.float() if k in ("q", "k", "v") else v) for k, v in x.items()}
    hv = sh.v.stop - sh.v.start
    rule = GatedDeltaRule(chunk_size=w.chunk)
    out = torch.empty(x["v"].shape, dtype=torch.float32, device=dev)
    st_out = torch.empty(w.n_seqs, hv, w.d_k, w.d_v, dtype=torch.float32, device=dev)

    def step():
        rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], None, out=out, state_out=st_out)

    k = max(1, min(args.steps, 5))
    total, per = timed(step, k, 1, dist, stream)
    ms = total / k
    return {"value": w.tokens / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "dtype": "f32", "kernel": "chunked_f32_d128 (f32 FMA)",
            "gpu_launches": k * rule.chunked_launches(x["q"], x["v"]),
            "tflops": prefill_flops(w, hv) / (statistics.mean(per) * 1e-3) / 1e12}


def bench_e2e(w, x, rule, out, st_out, args, dist, dev, stream) -> dict:
    """The same rule through the public host-buffer call (``gdr_chunked_host``):
    each step copies every input from pinned host memory to the GPU, runs, and
    copies the outputs and final states back, groups of sequences in flight so
    the copies in, the kernels and the copies out overlap."""
    host = {k: v.to("cpu").pin_memory() for k, v in x.items()}
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    st_h = torch.empty(st_out.shape, dtype=st_out.dtype).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_h.numel() * out_h.element_size() + st_h.numel() * st_h.element_size()

    def step():
        rule.chunked_host(host["q"], host["k"], host["v"], host["g"], host["beta"],
                          host.get("state"), cu_seqlens=host.get("cu_seqlens"), out=out_h,
                          state_out=st_h, device=dev, synchronize=False)

    k = max(1, min(args.steps, 5))
    total, _ = timed(step, k, 1, dist, stream)
    return {"value": w.tokens / (total / k * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}


L2_BYTES = 126 * 2**20  # B200


def l2_note(state_bytes_per_rank: float) -> str:
    """Whether a rank's share of a state pool updated in place step after
    step can stay in L2 between steps (no flush is done)."""
    mb = state_bytes_per_rank / 2**20
    if state_bytes_per_rank > L2_BYTES:
        return f"states {mb:.0f} MiB per rank, larger than L2 (126 MiB): streamed from HBM"
    return (f"states {mb:.0f} MiB per rank fit in L2 (126 MiB): consecutive steps may "
            "hit L2, as a decode loop of this size does")


def bench_decode(args, dist, dev, stream, pk, pk_kind) -> dict:
    w = workloads.get("decode")
    sh = shard_of(w, dist)
    x = sh.take(workloads.make_inputs(w, dev, seed=77))
    hq, hv = sh.qk.stop - sh.qk.start, sh.v.stop - sh.v.start
    steps_per = 64
    gen = torch.Generator(device=dev).manual_seed(5)

    def jitter(t):
        return (t + 0.01 * torch.randn(t.shape, generator=gen, device=dev).to(t.dtype))

    seq = {k: torch.stack([x[k]] + [jitter(x[k]) for _ in range(steps_per - 1)])
           for k in ("q", "k", "v", "g", "beta")}
    seq["g"] = seq["g"].clamp(max=0.0)
    seq["beta"] = seq["beta"].clamp(0.0, 1.0)
    states = x["state"]
    out = torch.empty(w.n_seqs, 1, hv, w.d_v, dtype=w.dtype, device=dev)
    rule = GatedDeltaRule()

    def steps():  # 64 consecutive decode steps, states in place
        for i in range(steps_per):
            rule.recurrent(seq["q"][i], seq["k"][i], seq["v"][i], seq["g"][i], seq["beta"][i],
                           states, out=out, state_out=states)

    # The 64 steps are captured once in a CUDA graph and replayed per step.
    steps()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        steps()
    step = graph.replay

    k = max(1, min(args.steps, 10))
    total, per = timed(step, k, max(3, args.warmup), dist, stream)
    ms = total / k / steps_per
    state_rw = 2.0 * w.n_seqs * w.heads_v * w.d_k * w.d_v * 4  # all ranks
    io = w.n_seqs * (w.heads_qk * w.d_k * 2 * 2 + w.heads_v * w.d_v * 2 * 2 + w.heads_v * 8)
    kern_ms = statistics.mean(per) / steps_per
    local_bytes = (state_rw + io) / dist.world
    del graph
    return {"metric": "decode state-update GB/s", "value": state_rw / (ms * 1e-3) / 1e9,
            "unit": "GB/s", "ms_per_step": ms, "steps_timed": k * steps_per, "cuda_graph": True,
            "gpu_launches": k * steps_per,
            "config": {"workload": "decode", "rows": w.n_seqs, "heads_qk": w.heads_qk,
                       "heads_v": w.heads_v, "d": w.d_k, "state_bytes_rw": state_rw,
                       "l2": l2_note(state_rw / 2 / dist.world)},
            "roofline": {"bound": "hbm", "achieved": local_bytes / (kern_ms * 1e-3) / 1e9,
                         "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": local_bytes / (kern_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                         "traffic": None, "peak_source": pk_kind}}


def bench_mixed(args, dist, dev, stream, pk, pk_kind) -> dict:
    w = workloads.get("mixed")
    sh = shard_of(w, dist)
    x = sh.take(workloads.make_inputs(w, dev, seed=55))
    hq, hv = sh.qk.stop - sh.qk.start, sh.v.stop - sh.v.start
    pool = x["state"]  # slot s = sequence s; updated in place every step
    rule = GatedDeltaRule()
    out = torch.empty_like(x["v"])
    import ctypes

    need = _lib.load().gdr_mixed_workspace_size(ctypes.byref(rule.params(x["q"], x["v"],
                                                                         x["cu_seqlens"])))
    ws = torch.empty(max(4, need), dtype=torch.uint8, device=dev)

    def step():
        rule.mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], pool, cu_seqlens=x["cu_seqlens"],
                   out=out, workspace=ws)

    total, per = timed(step, args.steps, args.warmup, dist, stream)
    ms = total / args.steps
    pre = [L for L in w.seqlens if L > 1]
    n_dec = sum(1 for L in w.seqlens if L == 1)
    pw = workloads.Workload("pre", tuple(pre), w.heads_qk, w.heads_v, w.d_k, w.d_v, w.chunk,
                            w.dtype, True, True)
    dec_bytes = n_dec * (2.0 * hv * w.d_k * w.d_v * 4
                         + hq * w.d_k * 4 + hv * w.d_v * 4 + hv * 8)
    nbytes = prefill_bytes(pw, hq, hv) + dec_bytes
    flops = prefill_flops(pw, hv)
    return {"metric": "mixed continuous batch, ms per launch", "value": ms, "unit": "ms",
            "higher_is_better": False, "tokens": w.tokens, "prefill_tokens": sum(pre),
            "decode_rows": n_dec, "gpu_launches": 2 * args.steps,
            "roofline": roofline(flops, nbytes, statistics.mean(per), pk, pk_kind, None)}


def bench_layer(args, dist, dev, stream, pk, pk_kind) -> dict:
    """The layer's steps around the rule on this rank's heads of the ragged
    pack: the causal conv with silu and the q/k/v split (4 taps, f32 states,
    HBM-bound), the prefill with the gates and gated norm fused, against the
    plain prefill, and the decode pool's row reorder (HBM-bound)."""
    from bunsen_b200.layer import causal_conv1d, gated_norm, state_reorder

    w = workloads.get("ragged_prefill")
    sh = shard_of(w, dist)
    hq, hv = sh.qk.stop - sh.qk.start, sh.v.stop - sh.v.start
    gen = torch.Generator(device=dev).manual_seed(61)
    t, n = w.tokens, w.n_seqs
    cu = torch.tensor([0] + list(np.cumsum(w.seqlens)), dtype=torch.int32, device=dev)
    res = {}

    # Conv: x [T, C] bf16, C = 2 H_qk d_k + H_v d_v channels of this rank.
    c, taps = 2 * hq * w.d_k + hv * w.d_v, 4
    x = torch.randn(t, c, device=dev, generator=gen).bfloat16()
    wt = (torch.randn(c, taps, device=dev, generator=gen) * 0.5).bfloat16()
    st = torch.randn(n, taps - 1, c, device=dev, generator=gen).bfloat16().float()
    st_out = torch.empty_like(st)
    splits = (hq * w.d_k, 2 * hq * w.d_k)

    def conv_step():
        causal_conv1d(x, wt, st, cu_seqlens=cu, silu=True, splits=splits, state_out=st_out)

    total, per = timed(conv_step, args.steps, args.warmup, dist, stream)
    nbytes = 2 * t * c * 2 + 2 * st.numel() * 4 + wt.numel() * 2
    ms = total / args.steps
    res["conv"] = {"value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
                   "channels": c, "taps": taps, "bytes_per_step": nbytes,
                   "roofline": roofline(0.0, nbytes, statistics.mean(per), pk, pk_kind, None)}
    del x, st, st_out

    # Prefill with the layer's gates and gated norm fused, against the plain one.
    full = workloads.make_inputs(w, dev, seed=1234)
    xin = sh.take(full)
    del full
    a = torch.randn(t, hv, device=dev, generator=gen).bfloat16()
    b = torch.randn(t, hv, device=dev, generator=gen).bfloat16()
    a_log = torch.log(torch.rand(hv, device=dev, generator=gen) * 0.2 + 0.01)
    dt_bias = torch.randn(hv, device=dev, generator=gen) * 0.1
    z = torch.randn(t, hv, w.d_v, device=dev, generator=gen).bfloat16()
    nw = torch.rand(w.d_v, device=dev, generator=gen) + 0.5
    rule = GatedDeltaRule(chunk_size=w.chunk)
    out = torch.empty(t, hv, w.d_v, dtype=torch.bfloat16, device=dev)
    so = torch.empty(n, hv, w.d_k, w.d_v, dtype=torch.float32, device=dev)

    def fused_step():
        rule.chunked(xin["q"], xin["k"], xin["v"], None, None, xin["state"], cu_seqlens=cu,
                     out=out, state_out=so, gates=(a, b, a_log, dt_bias), norm=(z, nw, 1e-6))

    def plain_step():
        rule.chunked(xin["q"], xin["k"], xin["v"], xin["g"], xin["beta"], xin["state"],
                     cu_seqlens=cu, out=out, state_out=so)

    def gates_then_norm_step():
        rule.chunked(xin["q"], xin["k"], xin["v"], None, None, xin["state"], cu_seqlens=cu,
                     out=out, state_out=so, gates=(a, b, a_log, dt_bias))
        gated_norm(out, z, nw, 1e-6, out=out)

    tf, _ = timed(fused_step, args.steps, args.warmup, dist, stream)
    ts, _ = timed(gates_then_norm_step, args.steps, args.warmup, dist, stream)
    tp, _ = timed(plain_step, args.steps, args.warmup, dist, stream)
    res["prefill_gates_norm"] = {"value": t / (tf / args.steps * 1e-3), "unit": "tokens/s",
                                 "ms_per_step": tf / args.steps,
                                 "separate_norm_ms_per_step": ts / args.steps,
                                 "plain_ms_per_step": tp / args.steps}
    del xin, a, b, z, out, so

    # Reorder of the decode workload's state pool (rows permuted).
    wd = workloads.get("decode")
    pool = torch.randn(wd.n_seqs, hv, w.d_k, w.d_v, device=dev, generator=gen)
    dst = torch.empty_like(pool)
    src = torch.randperm(wd.n_seqs, generator=gen, device=dev).to(torch.int32)

    def reorder_step():
        state_reorder(pool, src, out=dst)

    total, per = timed(reorder_step, args.steps, args.warmup, dist, stream)
    nbytes = 2 * pool.numel() * 4
    ms = total / args.steps
    res["reorder"] = {"value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
                      "rows": wd.n_seqs, "bytes_per_step": nbytes,
                      "roofline": roofline(0.0, nbytes, statistics.mean(per), pk, pk_kind, None)}
    res["gpu_launches"] = {"conv": 2 * args.steps, "reorder": args.steps}
    return res


def run_native(args, dist: Dist) -> None:
    torch.cuda.set_device(dist.local)
    dev = torch.device("cuda", dist.local)
    stream = torch.cuda.current_stream(dev)
    pk, pk_kind = peaks()
    lib = _lib.load()

    rag = bench_prefill("ragged_prefill", args, dist, dev, stream, pk, pk_kind, e2e=True,
                        verify=args.verify)
    dense = bench_prefill("dense_prefill", args, dist, dev, stream, pk, pk_kind)
    dense_f32 = bench_dense_f32(args, dist, dev, stream, pk, pk_kind)
    decode = bench_decode(args, dist, dev, stream, pk, pk_kind)
    mixed = bench_mixed(args, dist, dev, stream, pk, pk_kind)
    layer = bench_layer(args, dist, dev, stream, pk, pk_kind)
    if lib.gdr_device_error() != _lib.GDR_OK:
        raise RuntimeError("a kernel recorded a device-side failure")
    cpu = {}
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baselines()
    if dist.rank == 0:
        w = workloads.get("ragged_prefill")
        dense = {k: dense[k] for k in ("value", "unit", "ms_per_step", "roofline", "clocks")}
        dense["cpu_baseline"] = cpu.get("dense_prefill")
        dense_f32["cpu_baseline"] = cpu.get("dense_prefill")  # the oracle runs in f32
        decode["cpu_baseline"] = cpu.get("decode")
        mixed["cpu_baseline"] = cpu.get("mixed")
        line = {"metric": METRIC, "value": rag["value"], "unit": "tokens/s",
                "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": rag["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": headline_config(w, dist.world),
                "roofline": rag["roofline"], "cpu_baseline": cpu.get("ragged_prefill"),
                "e2e": rag["e2e"], "gpu_launches": rag["gpu_launches"], "clocks": rag["clocks"],
                "dense": dense, "dense_f32": dense_f32, "decode": decode, "mixed": mixed,
                "layer": layer}
        if "verified" in rag:
            line["verified"] = rag["verified"]
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--verify", action="store_true",
                    help="N > 1: check the gathered sharded outputs against one GPU")
    args = ap.parse_args()
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return
    dist.init()
    try:
        run_native(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
