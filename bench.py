#!/usr/bin/env python3
"""Benchmark of the B200 quantized GEMV hot path.

Default workload (the configuration BASELINE.json's metric is quoted on that
fits one GPU): Q8_0 GEMV on the Gemma-3 LM-head shape, 262144 x 640, batch 1,
seed 0.  A step is one GEMV over the whole weight.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl reference]

N > 1 is launched with torchrun (one process per GPU): the weight rows are
sharded over the ranks and the output slices are all-gathered (NCCL); the
total work is fixed, so scaling is "strong".  Timing: W untimed steps, then K
steps bracketed by barrier + synchronize, CUDA events on the library's stream,
max over ranks.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_0/Q8_0 GEMV HBM GB/s (% of ~8 TB/s) at 1/2/4/8 GPU; Gemma-3-270M decode tok/s"
UNIT = "GB/s"


def algorithmic_bytes(dtype: int, rows: int, cols: int, batch: int = 1) -> int:
    """Packed weight bytes + fp32 x + fp32 y of one GEMV (per-unit figures of
    the measurement table: e.g. 189,794,816 B for the Q8_0 LM head)."""
    from sapphire_b200 import row_bytes
    return rows * row_bytes(dtype, cols) + 4 * cols * batch + 4 * rows * batch


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.out.flush()
        self.out.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.out.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clocks unavailable"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- peaks / ncu --
def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "of measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "of fallback"}


def ncu_traffic(kernel_tag: str):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    p = os.path.join(ROOT, "profiles", f"{kernel_tag}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        line = line.strip()
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip().split()[0]))
            except ValueError:
                return None
    return None


# ---------------------------------------------------------- workload setup --
def build_weight(sp, ctx, cfg, seed=0):
    """Packed host bytes of the config's weight (GPU quantiser / packer) and x."""
    from sapphire_b200 import workloads
    src, X = workloads.make_inputs(cfg, seed=seed)
    if cfg.dtype == sp.DTYPE_TQ2_0:
        trits, scales = src
        packed = sp.pack_tq2(ctx, trits, scales)
    else:
        packed = sp.quantize(ctx, cfg.dtype, src)
    del src
    return packed, X


def cpu_reference_time(cfg, packed, X, budget_s: float, threads: int):
    """Reference kernel_gemv (oracle/_ref, the reference's own sources) on the
    host cores: seconds per call over a bounded number of calls."""
    from oracle.oracle import Reference, available_reference
    from sapphire_b200 import workloads
    if not available_reference():
        return None
    ref = Reference()
    ctx = ref.ctx(threads)
    t = ref.view(cfg.dtype, cfg.rows, cfg.cols, packed)
    xp = np.ascontiguousarray(workloads.pad_cols(X[:1], cfg.cols)[0])
    y = np.zeros(cfg.rows, dtype=np.float32)
    ref.L.kernel_gemv(ctx, y.ctypes.data, t, xp.ctypes.data)           # warm
    n, t0 = 0, time.perf_counter()
    while True:
        ref.L.kernel_gemv(ctx, y.ctypes.data, t, xp.ctypes.data)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s and n >= 3:
            break
    ref.L.tensor_release(t)
    ref.L.kernel_ctx_destroy(ctx)
    return el / n, n


def cpu_port_time(cfg, packed, X, budget_s: float, threads: int):
    """Oracle port (no reference kernel exists, e.g. ternary)."""
    from oracle.oracle import Oracle
    from sapphire_b200 import workloads
    o = Oracle()
    xp = workloads.pad_cols(X[:1], cfg.cols)
    n, t0 = 0, time.perf_counter()
    while True:
        o.gemv(cfg.dtype, packed, cfg.rows, cfg.cols, xp, nthreads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s and n >= 2:
            break
    return el / n, n


def cpu_baseline(cfg, packed, X, budget_s=12.0):
    threads = os.cpu_count() or 1
    per_call_bytes = algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols, 1)
    if cfg.dtype in (3, 4):
        r = cpu_reference_time(cfg, packed, X, budget_s, threads)
        kind = "reference"
    else:
        r = None
        kind = "port"
    if r is None:
        r = cpu_port_time(cfg, packed, X, budget_s, threads)
        kind = "port"
    sec, n = r
    return {"value": round(per_call_bytes / sec / 1e9, 3), "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{n} full {cfg.rows}x{cfg.cols} GEMV calls (batch 1), {sec * 1e3:.2f} ms each, "
                      f"{'reference kernel_gemv thread pool' if kind == 'reference' else 'oracle C port'} "
                      f"with {threads} threads"}


# ------------------------------------------------------------------ arms ----
def run_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import sapphire_b200 as sp
    from oracle.oracle import Oracle
    from sapphire_b200 import workloads
    # Quantise with the oracle quantiser (same bytes as the GPU quantiser) so
    # this arm needs no GPU.
    src, X = workloads.make_inputs(cfg, seed=0)
    o = Oracle()
    packed = o.pack_tq2(*src) if cfg.dtype == sp.DTYPE_TQ2_0 else o.quantize(cfg.dtype, src)
    del src
    threads = os.cpu_count() or 1
    bytes_per = algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols)
    fn = cpu_reference_time if cfg.dtype in (3, 4) else cpu_port_time
    kind = "reference" if cfg.dtype in (3, 4) else "port"
    # warm-up steps then timed steps, each one full GEMV call
    fn(cfg, packed, X, 0.0, threads) if args.warmup else None
    per = []
    for _ in range(args.steps):
        sec, _n = fn(cfg, packed, X, 0.0, threads)
        per.append(sec)
    sec = float(np.mean(per))
    value = bytes_per / sec / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 4),
            "higher_is_better": True, "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (PCG64 seed 0)",
            "config": {"workload": cfg.name, "rows": cfg.rows, "cols": cfg.cols, "format": sp.DTYPE_NAMES[cfg.dtype],
                       "parallelism": "host thread pool"},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": f"{args.steps} timed full GEMV calls after {args.warmup} warm-up"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_gpu_arm(args, cfg):
    import torch
    import torch.distributed as dist
    import sapphire_b200 as sp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    ctx = sp.Context(num_threads=1, device=local)
    if world > 1:
        uid = torch.zeros(sp.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(sp.shard_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        ctx.shard(rank, world, bytes(uid.cpu().numpy().tobytes()))

    # Two copies of the weight (different seeds) alternate between steps so
    # each step streams its weight from HBM (2 x 189.8 MB > 126 MB L2).
    packed0, X = build_weight(sp, ctx, cfg, seed=0)
    packed1, _ = build_weight(sp, ctx, cfg, seed=1)
    A = [sp.Tensor(cfg.dtype, (cfg.rows, cfg.cols), packed0), sp.Tensor(cfg.dtype, (cfg.rows, cfg.cols), packed1)]
    for a in A:
        ctx.check(sp.lib.kernel_tensor_upload(ctx.handle, a.handle), "upload")

    stream = torch.cuda.ExternalStream(ctx.stream)
    x_dev = torch.from_numpy(np.ascontiguousarray(X[:1])).cuda()
    y_dev = torch.zeros((1, cfg.rows), device="cuda")
    bytes_per = algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols, 1)

    def step(i):
        return sp.lib.kernel_gemv_device(ctx.handle, y_dev.data_ptr(), A[i & 1].handle, x_dev.data_ptr())

    for i in range(args.warmup):
        ctx.check(step(i), "warm-up")
    ctx.synchronize()

    # ---- device-timed region (value): K steps, events per step on the lib stream
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    # The clock sampler starts before the barrier so that every rank enters
    # the timed region together.
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ctx.synchronize()
    # Steps run back to back (no event between them), so with programmatic
    # dependent launch a step's weight stream may start under the tail of the
    # previous one, as in a serving loop.
    t_all0.record(stream)
    for i in range(args.steps):
        ctx.check(step(i), "step")
    t_all1.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    if world > 1:
        dist.barrier()
    total_ms = t_all0.elapsed_time(t_all1)
    # Per-launch duration of the GEMV alone (events around each launch).
    for i in range(args.steps):
        starts[i].record(stream)
        ctx.check(step(i), "step")
        ends[i].record(stream)
    ctx.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    t = torch.tensor([total_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = bytes_per / (ms_per_step * 1e-3) / 1e9

    # ---- dominant kernel duration (GEMV alone), for the roofline
    # (sharded: the timed call is the local GEMV followed by the all-gather)
    kern_ms = float(np.mean(step_ms))

    # ---- end-to-end through the public API with pinned host buffers
    x_host = torch.from_numpy(np.ascontiguousarray(X[:1])).pin_memory()
    y_host = torch.zeros((1, cfg.rows)).pin_memory()

    def e2e_step(i):
        return sp.lib.kernel_gemv(ctx.handle, y_host.data_ptr(), A[i & 1].handle, x_host.data_ptr())

    for i in range(args.warmup):
        ctx.check(e2e_step(i), "e2e warm-up")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    w0 = time.perf_counter()
    for i in range(args.steps):
        ctx.check(e2e_step(i), "e2e step")
    ev1.record(stream)
    ctx.synchronize()
    wall = time.perf_counter() - w0
    e2e_ms = max(ev0.elapsed_time(ev1), wall * 1e3)
    t = torch.tensor([e2e_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / args.steps
    e2e_value = bytes_per / (e2e_ms * 1e-3) / 1e9

    result = None
    if rank == 0:
        peaks = measured_peaks()
        # achieved: algorithmic bytes of one launch (this rank's rows) / launch time
        per_rank_rows = (cfg.rows + world - 1) // world if world > 1 else cfg.rows
        kern_bytes = algorithmic_bytes(cfg.dtype, per_rank_rows, cfg.cols, 1)
        achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
        tag = f"gemv_{sp.DTYPE_NAMES[cfg.dtype].lower()}_{cfg.name}"
        clocks = sampler.summary() if sampler else {}
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (PCG64 seed 0; N(0,0.02) weights quantised on the GPU, N(0,1) x)",
            "config": {"workload": cfg.name, "rows": cfg.rows, "cols": cfg.cols,
                       "format": sp.DTYPE_NAMES[cfg.dtype], "batch": 1,
                       "parallelism": f"row-shard x{world} + NCCL all-gather" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: two weight copies alternate between steps",
                       "algorithmic_bytes_per_step": bytes_per},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "kernel_ms": round(kern_ms, 5), "traffic": ncu_traffic(tag), "kernel": tag,
                         "kernel_ms_covers": "GEMV kernel" if world == 1 else "local GEMV + NCCL all-gather"},
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": 4 * cfg.cols,
                    "d2h_bytes_per_step": 4 * cfg.rows, "ms_per_step": round(e2e_ms, 5),
                    "path": "kernel_gemv with pinned host x/y (weights resident after upload)"},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(cfg, packed0, X)
    for a in A:
        a.release()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


# ------------------------------------------------------------- prefill ------
PREFILL_METRIC = "Q4_0 prefill dequant-GEMM TFLOP/s (tcgen05 tensor cores)"
PREFILL_UNIT = "TFLOP/s"


def prefill_flops(cfg, tokens=None) -> int:
    return 2 * (cfg.batch if tokens is None else tokens) * cfg.rows * cfg.cols


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def cpu_prefill_time(cfg, packed, X, tokens: int, threads: int):
    """Seconds for `tokens` reference kernel_gemv calls (one per token, the
    reference's prefill; its Q4_0 kernel_gemm returns -1) on bf16-rounded
    activations.  Falls back to the oracle port without oracle/_ref."""
    from oracle.oracle import Reference, Oracle, available_reference
    from sapphire_b200 import workloads
    xs = workloads.pad_cols(bf16_round(X[:tokens]), cfg.cols)
    if available_reference():
        ref = Reference()
        ctx = ref.ctx(threads)
        t = ref.view(cfg.dtype, cfg.rows, cfg.cols, packed)
        y = np.zeros(cfg.rows, dtype=np.float32)
        ref.L.kernel_gemv(ctx, y.ctypes.data, t, xs[0].ctypes.data)          # warm
        t0 = time.perf_counter()
        for i in range(tokens):
            ref.L.kernel_gemv(ctx, y.ctypes.data, t, xs[i].ctypes.data)
        el = time.perf_counter() - t0
        ref.L.tensor_release(t)
        ref.L.kernel_ctx_destroy(ctx)
        return el, "reference"
    o = Oracle()
    t0 = time.perf_counter()
    o.gemv(cfg.dtype, packed, cfg.rows, cfg.cols, xs, nthreads=threads)
    return time.perf_counter() - t0, "port"


def prefill_cpu_baseline(cfg, packed, X, budget_s=10.0):
    threads = os.cpu_count() or 1
    el, kind = cpu_prefill_time(cfg, packed, X, 4, threads)
    tokens = int(max(4, min(cfg.batch, 4 * budget_s / max(el, 1e-6))))
    el, kind = cpu_prefill_time(cfg, packed, X, tokens, threads)
    return {"value": round(prefill_flops(cfg, tokens) / el / 1e12, 5), "unit": PREFILL_UNIT, "cores": threads,
            "kind": kind,
            "sample": f"{tokens} of the {cfg.batch} tokens, one {'reference kernel_gemv' if kind == 'reference' else 'oracle port GEMV'}"
                      f" call per token ({el / tokens * 1e3:.2f} ms each) with {threads} threads"}


def run_reference_prefill(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import sapphire_b200 as sp
    from oracle.oracle import Oracle
    from sapphire_b200 import workloads
    src, X = workloads.make_inputs(cfg, seed=0)
    packed = Oracle().quantize(cfg.dtype, src)
    del src
    threads = os.cpu_count() or 1
    tokens = 8                                   # per step: a bounded sample of the 2048 tokens
    for _ in range(args.warmup):
        cpu_prefill_time(cfg, packed, X, 1, threads)
    total, kind = 0.0, "reference"
    for _ in range(args.steps):
        el, kind = cpu_prefill_time(cfg, packed, X, tokens, threads)
        total += el
    value = prefill_flops(cfg, tokens) * args.steps / total / 1e12
    line = {"impl": "reference", "metric": PREFILL_METRIC, "value": round(value, 5), "unit": PREFILL_UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (PCG64 seed 0)",
            "config": {"workload": cfg.name, "rows": cfg.rows, "cols": cfg.cols, "tokens": cfg.batch,
                       "format": "Q4_0", "parallelism": "host thread pool"},
            "cpu_baseline": {"value": round(value, 5), "unit": PREFILL_UNIT, "cores": threads, "kind": kind,
                             "sample": f"each step {tokens} of the {cfg.batch} tokens, one kernel_gemv per token"},
            "e2e": {"value": round(value, 5), "unit": PREFILL_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_gpu_prefill(args, cfg):
    import torch
    import torch.distributed as dist
    import sapphire_b200 as sp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = sp.Context(num_threads=1, device=local)
    if world > 1:
        uid = torch.zeros(sp.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(sp.shard_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        ctx.shard(rank, world, bytes(uid.cpu().numpy().tobytes()))

    packed0, X = build_weight(sp, ctx, cfg, seed=0)
    packed1, X1 = build_weight(sp, ctx, cfg, seed=1)
    A = [sp.Tensor(cfg.dtype, (cfg.rows, cfg.cols), packed0), sp.Tensor(cfg.dtype, (cfg.rows, cfg.cols), packed1)]
    for a in A:
        ctx.check(sp.lib.kernel_tensor_upload(ctx.handle, a.handle), "upload")
    stream = torch.cuda.ExternalStream(ctx.stream)
    Xd = [torch.from_numpy(np.ascontiguousarray(X)).cuda(), torch.from_numpy(np.ascontiguousarray(X1)).cuda()]
    Yd = torch.zeros((cfg.batch, cfg.rows), device="cuda")
    flops = prefill_flops(cfg)

    def step(i):
        return sp.lib.kernel_gemm_device(ctx.handle, Yd.data_ptr(), A[i & 1].handle, Xd[i & 1].data_ptr(), cfg.batch)

    for i in range(args.warmup):
        ctx.check(step(i), "warm-up")
    ctx.synchronize()
    t0e = torch.cuda.Event(enable_timing=True)
    t1e = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0e.record(stream)
    for i in range(args.steps):
        ctx.check(step(i), "step")
    t1e.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    if world > 1:
        dist.barrier()
    t = torch.tensor([t0e.elapsed_time(t1e)], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    value = flops / (ms_per_step * 1e-3) / 1e12

    # GEMM kernel alone (activations already bf16 on the device), unsharded.
    kern_ms = None
    if world == 1:
        kp = ((cfg.cols + 31) // 32 * 32 + 63) // 64 * 64
        Xb = []
        for x in Xd:
            xb = torch.zeros((cfg.batch, kp), dtype=torch.bfloat16, device="cuda")
            xb[:, :cfg.cols] = x.to(torch.bfloat16)
            Xb.append(xb)
        torch.cuda.synchronize()

        def kstep(i):
            return sp.lib.kernel_gemm_device_bf16(ctx.handle, Yd.data_ptr(), A[i & 1].handle, Xb[i & 1].data_ptr(),
                                                  cfg.batch, kp)
        for i in range(args.warmup):
            ctx.check(kstep(i), "kernel warm-up")
        ctx.synchronize()
        evs = []
        for i in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ctx.check(kstep(i), "kernel step")
            e1.record(stream)
            evs.append((e0, e1))
        ctx.synchronize()
        kern_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))

    # End to end through kernel_gemm with pinned host buffers (X in, Y out).
    xh = [torch.from_numpy(np.ascontiguousarray(X)).pin_memory(), torch.from_numpy(np.ascontiguousarray(X1)).pin_memory()]
    yh = torch.zeros((cfg.batch, cfg.rows)).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step(i):
        return sp.lib.kernel_gemm(ctx.handle, yh.data_ptr(), A[i & 1].handle, xh[i & 1].data_ptr(), cfg.batch,
                                  cfg.rows)
    for i in range(args.warmup):
        ctx.check(e2e_step(i), "e2e warm-up")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    w0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.check(e2e_step(i), "e2e step")
    ev1.record(stream)
    ctx.synchronize()
    e2e_ms = max(ev0.elapsed_time(ev1), (time.perf_counter() - w0) * 1e3)
    t = torch.tensor([e2e_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / e2e_steps

    result = None
    if rank == 0:
        peaks = measured_peaks()
        tag = f"gemm_tc_{cfg.name}"
        roof = {"bound": "tensor", "unit": PREFILL_UNIT, "peak": peaks["bf16_tflops"],
                "peak_source": peaks["source"] + " (dense bf16 cuBLAS, burst)", "kernel": tag,
                "traffic": ncu_traffic(tag),
                "note": "achieved counts the algorithmic 2*tokens*rows*cols FLOP; the kernel issues twice as "
                        "many MMA FLOP (hi + lo weight halves)"}
        if kern_ms is not None:
            ach = flops / (kern_ms * 1e-3) / 1e12
            roof.update({"achieved": round(ach, 2), "frac": round(ach / peaks["bf16_tflops"], 4),
                         "kernel_ms": round(kern_ms, 5)})
        else:
            roof.update({"achieved": None, "frac": None, "kernel_ms": None})
        result = {
            "metric": PREFILL_METRIC, "value": round(value, 3), "unit": PREFILL_UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (PCG64 seed 0; N(0,0.02) weights quantised on the GPU, N(0,1) X)",
            "config": {"workload": cfg.name, "rows": cfg.rows, "cols": cfg.cols, "tokens": cfg.batch,
                       "format": "Q4_0", "parallelism": f"row-shard x{world} + NCCL all-gather" if world > 1
                       else "single GPU", "flop_per_step": flops,
                       "l2": "inputs larger than L2: 84 MB of Y written per step, weights and X alternate"},
            "roofline": roof,
            "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": PREFILL_UNIT,
                    "h2d_bytes_per_step": 4 * cfg.batch * cfg.cols, "d2h_bytes_per_step": 4 * cfg.batch * cfg.rows,
                    "ms_per_step": round(e2e_ms, 4), "path": "kernel_gemm with pinned host X/Y"},
            "gpu_launches": 2 * args.steps,
            "clocks": sampler.summary() if sampler else {},
        }
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = prefill_cpu_baseline(cfg, packed0, X)
    for a in A:
        a.release()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


# -------------------------------------------------------------- decode -----
DECODE_METRIC = "Gemma-3-270M decode tok/s (greedy, Q4_0 projections and LM head)"
DECODE_UNIT = "tok/s"


def decode_bytes_per_token(cfg, pos: int) -> int:
    """Algorithmic HBM bytes of one generated token at position `pos`: every
    packed Q4_0 projection and the LM head, the embedding row, the KV rows the
    attention reads (the window for local layers) and writes, x/y vectors
    neglected (< 0.1 %)."""
    from sapphire_b200 import row_bytes
    w = 0
    for _, rows, cols in cfg.projections():
        w += rows * row_bytes(3, cols)
    w *= cfg.layers
    w += cfg.vocab * row_bytes(3, cfg.hidden) + 2 * cfg.hidden
    kv_row = cfg.kv_heads * cfg.head_dim * 4
    for layer in range(cfg.layers):
        n = pos + 1 if cfg.is_global(layer) else min(pos + 1, cfg.sliding_window)
        w += 2 * n * kv_row + 2 * kv_row
    return w


def decode_cpu_baseline(cfg, model, n_gen=None):
    from oracle.oracle import ReferenceDecode, available_reference_decode
    if not available_reference_decode():
        return None
    toks, _, _, tp, td = ReferenceDecode().run(cfg, model, n_gen=n_gen)
    n = len(toks)
    return {"value": round(n / td, 3), "unit": DECODE_UNIT, "cores": os.cpu_count() or 1, "kind": "reference",
            "sample": f"one reference decode (its inference_forward per token, Q4_0 kernel_gemv, all host "
                      f"threads): {cfg.prompt}-token prompt in {tp:.1f} s, then {n} greedy tokens in {td:.2f} s"}


def run_reference_decode(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.oracle import Oracle, available_reference_decode
    from sapphire_b200 import workloads
    if not available_reference_decode():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdecode_ref.so not built "
                          "(make -C oracle ref needs the reference sources)"}), flush=True)
        return 0
    o = Oracle()
    model = workloads.make_decode_model(cfg, lambda a: o.quantize(3, a), seed=0)
    n_gen = max(1, min(args.steps, cfg.generate))
    cb = decode_cpu_baseline(cfg, model, n_gen=n_gen)
    line = {"impl": "reference", "metric": DECODE_METRIC, "value": cb["value"], "unit": DECODE_UNIT,
            "n_gpus": args.gpus, "steps": n_gen, "warmup": 0, "ms_per_step": round(1e3 / cb["value"], 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (PCG64 seed 0, random-init Gemma-3-270M)",
            "config": {"workload": cfg.name, "prompt": cfg.prompt, "generated": n_gen,
                       "parallelism": "host thread pool"},
            "cpu_baseline": dict(cb, sample=cb["sample"] + "; a step is one generated token"),
            "e2e": {"value": cb["value"], "unit": DECODE_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_gpu_decode(args, cfg):
    """Each step is one full request: the 512-token prompt, then 64 greedy
    tokens.  `value` is generated tokens per second of the generation phase
    (device events); N > 1 runs independent replicas (decode does not shard)."""
    import torch
    import torch.distributed as dist
    import sapphire_b200 as sp
    from sapphire_b200 import workloads
    from sapphire_b200.decode import Decoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    ctx = sp.Context(num_threads=1, device=local)
    model = workloads.make_decode_model(cfg, lambda a: sp.quantize(ctx, 3, a), seed=0)
    dec = Decoder(ctx, cfg, model)
    prompt = model["prompt"]
    for _ in range(args.warmup):
        dec.generate(prompt, cfg.generate)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    gen_ms, prompt_ms, walls = [], [], []
    ids = None
    for _ in range(args.steps):
        w0 = time.perf_counter()
        ids, _ = dec.generate(prompt, cfg.generate)
        walls.append(time.perf_counter() - w0)
        pm, gm = dec.last_times()
        prompt_ms.append(pm)
        gen_ms.append(gm)
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    t = torch.tensor([float(np.sum(gen_ms)), float(np.sum(prompt_ms)), float(np.sum(walls))], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gen_total, prompt_total, wall_total = (float(v) for v in t.tolist())
    n_tok = cfg.generate * args.steps
    value = world * n_tok / (gen_total * 1e-3)
    result = None
    if rank == 0:
        peaks = measured_peaks()
        bpt = float(np.mean([decode_bytes_per_token(cfg, cfg.prompt - 1 + g) for g in range(cfg.generate)]))
        ms_tok = gen_total / n_tok
        achieved = bpt / (ms_tok * 1e-3) / 1e9
        golden = os.path.join(ROOT, "tests", "golden", "decode_gemma3_270m_seed0.npz")
        match = None
        if os.path.exists(golden):
            match = bool(np.array_equal(ids, np.load(golden)["tokens"]))
        result = {
            "metric": DECODE_METRIC, "value": round(value, 2), "unit": DECODE_UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(gen_total / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (PCG64 seed 0; random-init Gemma-3-270M, N(0,0.02) weights, Q4_0 projections "
                    "and LM head, bf16 embedding, zero norm weights)",
            "config": {"workload": cfg.name, "prompt": cfg.prompt, "generated": cfg.generate,
                       "context": cfg.context, "sliding_window": cfg.sliding_window,
                       "parallelism": f"{world} independent replicas" if world > 1 else "single GPU",
                       "step": "one request: prompt then greedy generation",
                       "l2": "inputs larger than L2: 168 MB of weights read per token",
                       "prompt_tok_s": round((cfg.prompt - 1) * args.steps / (prompt_total * 1e-3), 1),
                       "tokens_match_reference": match},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "kernel_ms": round(ms_tok, 5), "traffic": None,
                         "kernel": "decode step graph (generation phase, per token)",
                         "bytes_per_token": int(bpt)},
            "e2e": {"value": round(n_tok / wall_total, 2), "unit": DECODE_UNIT,
                    "h2d_bytes_per_step": 4 * cfg.prompt, "d2h_bytes_per_step": 8 * cfg.generate,
                    "ms_per_step": round(wall_total / args.steps * 1e3, 3),
                    "path": "sapphire_decoder_generate with a host prompt and host ids (prompt phase included)"},
            "gpu_launches": args.steps * (cfg.generate * dec.launches_per_token
                                          + (cfg.prompt - 1) * (dec.launches_per_token - 1)),
            "clocks": sampler.summary() if sampler else {},
        }
        if world == 1 and not args.no_cpu_baseline:
            cb = decode_cpu_baseline(cfg, model)
            if cb:
                result["cpu_baseline"] = cb
    dec.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="sapphire", choices=["sapphire", "reference"])
    ap.add_argument("--config", default="q8_0_lm_head_262144x640")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    from sapphire_b200 import workloads
    if args.config == workloads.C3.name:
        cfg = workloads.C3
        return run_reference_decode(args, cfg) if args.impl == "reference" else run_gpu_decode(args, cfg)
    cfg = workloads.CONFIGS[args.config]
    if cfg.batch > 1:
        return run_reference_prefill(args, cfg) if args.impl == "reference" else run_gpu_prefill(args, cfg)
    if args.impl == "reference":
        return run_reference_arm(args, cfg)
    return run_gpu_arm(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
