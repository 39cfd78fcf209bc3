#!/usr/bin/env python3
"""Benchmark of the gated delta rule on B200s.

One JSON line (rank 0). The headline `value` is ragged prefill tokens/s: one
step is one gdr_chunked call over the whole ragged pack (131072 tokens in 64
lognormal sequences, 16 q/k heads, 32 v heads, d 128, chunk 64, bf16, f32
states), inputs resident in HBM (2.3 GB, larger than L2, so no flush is
needed). The `decode` object carries the decode state-update figure: 64
consecutive single-token steps over 256 rows with f32 states [256, 32, 128,
128] updated in place.

With N GPUs (torchrun), the heads are sharded: rank r runs q/k heads
[r*16/N, (r+1)*16/N) with their v heads over the same pack; no data crosses
GPUs; the time is the maximum over ranks; `value` counts the pack's tokens
(all heads) once -- strong scaling.

`--impl reference` times the CPU oracle (a C++ restatement of bunsen's burn
rule, OpenMP over all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
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

METRIC = "GDR prefill tokens/sec (ragged) and decode state-update GB/s vs HBM peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------
def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def prefill_flops_per_token_head(c: int, d: int) -> float:
    """Algorithmic FLOPs per token per v-head: 10 C d + 6 d^2 + (2/3) C^2 (the
    chunk's matmuls: 5 C x C x d, 3 C x d x d, the C^3/3 inverse)."""
    return 10 * c * d + 6 * d * d + (2.0 / 3.0) * c * c


def prefill_bytes(w: workloads.Workload, heads_qk: int, heads_v: int) -> float:
    """Algorithmic HBM bytes of one prefill pass: q, k (once per q/k head),
    v, out in bf16, g and beta in f32, states read (if given) and written."""
    per_tok = heads_qk * w.d_k * 2 * 2 + heads_v * w.d_v * 2 * 2 + heads_v * 4 * 2
    states = w.n_seqs * heads_v * w.d_k * w.d_v * 4 * (2 if w.with_state else 1)
    return float(w.tokens * per_tok + states)


def shard(x: dict, w: workloads.Workload, rank: int, world: int) -> dict:
    """The q/k heads and v heads of rank `rank`."""
    hq0, hq1 = rank * w.heads_qk // world, (rank + 1) * w.heads_qk // world
    g = w.heads_v // w.heads_qk
    out = {}
    for k, t in x.items():
        if k in ("q", "k"):
            out[k] = t[..., hq0:hq1, :].contiguous()
        elif k in ("v",):
            out[k] = t[..., hq0 * g:hq1 * g, :].contiguous()
        elif k in ("g", "beta"):
            out[k] = t[..., hq0 * g:hq1 * g].contiguous()
        elif k == "state":
            out[k] = t[:, hq0 * g:hq1 * g].contiguous()
        else:
            out[k] = t
    return out


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
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
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
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
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

    def init(self, backend: str = "nccl"):
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local)
                                    if backend == "nccl" else None)
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
    synchronize on both sides; per-step CUDA events on the launching stream.
    Returns (max-over-ranks total ms, this rank's per-step ms)."""
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


# ---------------------------------------------------------------------------
def cpu_sample_prefill(w: workloads.Workload, seconds_hint: float = 15.0) -> dict:
    """The oracle's chunked form on a bounded sample of the ragged pack (the
    first sequences, up to ~8k tokens, at 8 of the 32 v heads), all host
    threads; tokens/s scaled to all heads."""
    from oracle import oracle

    lens, tot = [], 0
    for L in w.seqlens:
        if tot + L > 8192 and lens:
            break
        lens.append(L)
        tot += L
    heads_v, heads_qk = 8, 4
    sw = workloads.Workload("sample", tuple(lens), heads_qk, heads_v, w.d_k, w.d_v, w.chunk,
                            w.dtype, True, True)
    x = workloads.make_inputs(sw, "cpu", seed=99)
    f = {k: workloads.to_numpy_f32(v) for k, v in x.items() if k != "cu_seqlens"}
    cu = x["cu_seqlens"].numpy().astype(np.int32)
    threads = oracle.max_threads()
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.chunked(f["q"], f["k"], f["v"], f["g"], f["beta"], f["state"], cu_seqlens=cu,
                       chunk_size=w.chunk, threads=threads)
        reps += 1
        if time.perf_counter() - t0 > seconds_hint or reps >= 50:
            break
    dt = (time.perf_counter() - t0) / reps
    tok_s = tot * heads_v / w.heads_v / dt
    return {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{len(lens)} sequences / {tot} tokens at {heads_v} of {w.heads_v} v heads, "
                      f"{reps} reps; scaled to all heads"}


def run_reference(args, dist: Dist) -> None:
    if dist.rank != 0:
        return
    w = workloads.get("ragged_prefill")
    per = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        r = cpu_sample_prefill(w, seconds_hint=0.0)
        if i >= args.warmup:
            per.append(time.perf_counter() - t0)
    tok_s = r["value"]
    r["value"] = tok_s
    line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(per), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "ragged_prefill", "tokens": w.tokens, "n_seqs": w.n_seqs,
                       "heads_qk": w.heads_qk, "heads_v": w.heads_v, "d": w.d_k,
                       "chunk": w.chunk},
            "cpu_baseline": r,
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def run_native(args, dist: Dist) -> None:
    torch.cuda.set_device(dist.local)
    dev = torch.device("cuda", dist.local)
    stream = torch.cuda.current_stream(dev)
    pk, pk_kind = peaks()
    lib = _lib.load()

    # -- ragged prefill (the headline) --------------------------------------
    w = workloads.get("ragged_prefill")
    full = workloads.make_inputs(w, dev, seed=1234)
    x = shard(full, w, dist.rank, dist.world)
    del full
    hq, hv = x["q"].shape[1], x["v"].shape[1]
    rule = GatedDeltaRule(chunk_size=w.chunk)
    out = torch.empty(w.tokens, hv, w.d_v, dtype=w.dtype, device=dev)
    st_out = torch.empty(w.n_seqs, hv, w.d_k, w.d_v, dtype=torch.float32, device=dev)

    def prefill_step():
        rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                     cu_seqlens=x["cu_seqlens"], out=out, state_out=st_out)

    with Clocks(dist.local) as clk:
        total_ms, per = timed(prefill_step, args.steps, args.warmup, dist, stream)
    assert lib.gdr_device_error() == _lib.GDR_OK
    ms = total_ms / args.steps
    tok_s = w.tokens / (ms * 1e-3)
    kern_ms = statistics.mean(per)  # one launch per step: the kernel's duration
    flops = prefill_flops_per_token_head(w.chunk, w.d_k) * w.tokens * hv
    nbytes = prefill_bytes(w, hq, hv)
    t_flop = flops / (pk["bf16_tflops_sustained"] * 1e12)
    t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
    if t_flop >= t_hbm:
        ach, peak, unit = flops / (kern_ms * 1e-3) / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s"
        bound = "tensor"
    else:
        ach, peak, unit = nbytes / (kern_ms * 1e-3) / 1e9, pk["hbm_gbs"], "GB/s"
        bound = "hbm"
    roofline = {"bound": bound, "achieved": ach, "peak": peak, "unit": unit, "frac": ach / peak,
                "traffic": None, "peak_source": pk_kind,
                "attainable_frac": max(t_flop, t_hbm) / (kern_ms * 1e-3),
                "flops_per_launch": flops, "bytes_per_launch": nbytes,
                "tflops": flops / (kern_ms * 1e-3) / 1e12,
                "gbs": nbytes / (kern_ms * 1e-3) / 1e9}

    # -- end to end: host buffers through the public API ---------------------
    host = {k: v.to("cpu").pin_memory() for k, v in x.items()}
    dbuf = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    st_h = torch.empty(st_out.shape, dtype=st_out.dtype).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_h.numel() * out_h.element_size() + st_h.numel() * st_h.element_size()

    def e2e_step():
        for k, v in host.items():
            dbuf[k].copy_(v, non_blocking=True)
        rule.chunked(dbuf["q"], dbuf["k"], dbuf["v"], dbuf["g"], dbuf["beta"], dbuf["state"],
                     cu_seqlens=dbuf["cu_seqlens"], out=out, state_out=st_out)
        out_h.copy_(out, non_blocking=True)
        st_h.copy_(st_out, non_blocking=True)

    e2e_steps = max(1, min(args.steps, 5))
    e2e_ms, _ = timed(e2e_step, e2e_steps, 1, dist, stream)
    e2e = {"value": w.tokens / (e2e_ms / e2e_steps * 1e-3), "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    del host, dbuf, x

    # -- decode: 64 consecutive steps, states in place -----------------------
    wd = workloads.get("decode")
    steps_per = 64
    dx = shard(workloads.make_inputs(wd, dev, seed=77), wd, dist.rank, dist.world)
    hvd = dx["v"].shape[2]
    gen = torch.Generator(device=dev).manual_seed(5)
    seq = {k: torch.stack([dx[k]] + [
        (dx[k] + 0.01 * torch.randn(dx[k].shape, generator=gen, device=dev).to(dx[k].dtype))
        for _ in range(steps_per - 1)]) for k in ("q", "k", "v", "g", "beta")}
    seq["g"] = seq["g"].clamp(max=0.0)
    seq["beta"] = seq["beta"].clamp(0.0, 1.0)
    states = dx["state"]
    dout = torch.empty(wd.n_seqs, 1, hvd, wd.d_v, dtype=wd.dtype, device=dev)
    drule = GatedDeltaRule()

    def decode_step():
        for i in range(steps_per):
            drule.recurrent(seq["q"][i], seq["k"][i], seq["v"][i], seq["g"][i], seq["beta"][i],
                            states, out=dout, state_out=states)

    dsteps = max(1, min(args.steps, 10))
    d_total, d_per = timed(decode_step, dsteps, max(3, min(args.warmup, 3)), dist, stream)
    d_ms = d_total / dsteps / steps_per
    state_bytes = 2.0 * wd.n_seqs * hvd * wd.d_k * wd.d_v * 4 * dist.world
    io_bytes = wd.n_seqs * dist.world * (hq * wd.d_k * 2 * 2 + hvd * wd.d_v * 2 * 2 + hvd * 8)
    d_gbs = state_bytes / (d_ms * 1e-3) / 1e9
    d_kern_ms = statistics.mean(d_per) / steps_per
    per_gpu_bytes = (state_bytes + io_bytes) / dist.world
    decode = {"metric": "decode state-update GB/s", "value": d_gbs, "unit": "GB/s",
              "ms_per_step": d_ms, "steps_timed": dsteps * steps_per,
              "gpu_launches": dsteps * steps_per,
              "config": {"workload": "decode", "rows": wd.n_seqs, "heads_qk": wd.heads_qk,
                         "heads_v": wd.heads_v, "d": wd.d_k, "state_bytes_rw": state_bytes},
              "roofline": {"bound": "hbm", "achieved": per_gpu_bytes / (d_kern_ms * 1e-3) / 1e9,
                           "peak": pk["hbm_gbs"], "unit": "GB/s",
                           "frac": per_gpu_bytes / (d_kern_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                           "traffic": None, "peak_source": pk_kind}}
    del seq, states, dx

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_sample_prefill(w)

    if dist.rank == 0:
        line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": dist.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "ragged_prefill", "tokens": w.tokens, "n_seqs": w.n_seqs,
                           "max_len": max(w.seqlens), "heads_qk": w.heads_qk,
                           "heads_v": w.heads_v, "d": w.d_k, "chunk": w.chunk,
                           "parallelism": f"heads{dist.world}",
                           "l2": "inputs larger than L2 (no flush)"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": args.steps,
                "clocks": clk.summary(), "decode": decode}
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return
    dist.init("nccl")
    try:
        run_native(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
