#!/usr/bin/env python3
"""Benchmark of the B200 quantized GEMV hot path.

Default run (no --config): the headline line is the Q8_0 GEMV on the Gemma-3
LM-head shape, 262144 x 640, batch 1, seed 0 (the configuration BASELINE.json's
metric is quoted on that fits one GPU); a step is one GEMV over the whole
weight.  The same line carries a `secondary` object with every other
configuration of the metric measured in the same run: the Q4_0 and ternary
GEMVs on the LM-head shape, the ternary 16384 x 16384 GEMV, the tcgen05 Q4_0
prefill product and the Gemma-3-270M decode.  Each entry has its own value,
roofline, e2e, parity and (at N = 1) CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl reference]
                    [--no-secondary] [--no-cpu-baseline]

N > 1 is launched with torchrun (one process per GPU): the weight rows are
sharded over the ranks and every rank receives the whole output (peer-memory
gather from the GEMV epilogue for batch 1, NCCL all-gather for batched
products); the matrix is fixed, so scaling is "strong".  Decode does not
shard: N > 1 runs N independent replicas.  Timing: W untimed steps, then K
steps bracketed by barrier + synchronize, CUDA events on the library's stream,
max over ranks.  Rank 0 prints one JSON line.

Every measured configuration ends with a parity check outside the timed
region: the output of one more product against the oracle (the C restatement
of the reference row kernels, run in f64 on the host) and, at N > 1, a hash of
every rank's output compared across ranks.  A failed check exits non-zero.

`--impl reference` times the reference's own CPU implementation (its
kernel_gemv thread pool and AVX2 row kernels compiled unmodified into
oracle/_ref) on the same workload; it loads nothing of the GPU library.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_0/Q8_0 GEMV HBM GB/s (% of ~8 TB/s) at 1/2/4/8 GPU; Gemma-3-270M decode tok/s"
UNIT = "GB/s"
GEMV_RTOL = 1e-4          # normwise parity bar of the GEMV path


def load_workloads():
    """sapphire_b200/workloads.py loaded by file path, without importing the
    package (whose __init__ maps libsapphire_cuda.so): the reference arm must
    map nothing of the GPU library."""
    name = "sapphire_bench_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "sapphire_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


WL = load_workloads()


def algorithmic_bytes(dtype: int, rows: int, cols: int, batch: int = 1) -> int:
    """Packed weight bytes + fp32 x + fp32 y of one GEMV (per-unit figures of
    the measurement table: e.g. 189,794,816 B for the Q8_0 LM head)."""
    return rows * WL.row_bytes(dtype, cols) + 4 * cols * batch + 4 * rows * batch


def host_cpu() -> dict:
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count() or 1}


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled around the timed region
    (started before the warm-up steps, stopped after the timed steps)."""
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


class NoSampler:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        pass

    def summary(self) -> dict:
        return {}


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


# ------------------------------------------------- configuration records ----
# The `config` object is built by the same function in both arms so the two
# lines describe the same workload; how an arm executes it goes to the
# top-level `execution` key.
def gemv_config(cfg, world: int) -> dict:
    return {"workload": cfg.name, "rows": cfg.rows, "cols": cfg.cols, "format": WL.DTYPE_NAMES[cfg.dtype],
            "batch": 1, "parallelism": f"row-shard x{world}" if world > 1 else "single device",
            "l2": "weight larger than the 126 MB GPU L2 or two weight copies alternating between steps",
            "algorithmic_bytes_per_step": algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols)}


def prefill_config(cfg, world: int) -> dict:
    return {"workload": cfg.name, "rows": cfg.rows, "cols": cfg.cols, "tokens": cfg.batch, "format": "Q4_0",
            "parallelism": f"row-shard x{world}" if world > 1 else "single device",
            "flop_per_step": prefill_flops(cfg),
            "l2": "inputs larger than L2: 84 MB of Y written per step, weights and X alternate"}


def decode_config(cfg, world: int) -> dict:
    return {"workload": cfg.name, "prompt": cfg.prompt, "generated": cfg.generate, "context": cfg.context,
            "sliding_window": cfg.sliding_window,
            "parallelism": f"LM head row-sharded x{world} (8-byte argmax exchange)" if world > 1 else "single device",
            "step": "one request: prompt then greedy generation",
            "l2": "inputs larger than L2: 168 MB of weights read per token"}


# ------------------------------------------------------------- CPU side ------
def cpu_reference_time(cfg, packed, X, budget_s: float, threads: int):
    """Reference kernel_gemv (oracle/_ref, the reference's own sources) on the
    host cores: seconds per call over a bounded number of calls."""
    from oracle.oracle import Reference, available_reference
    if not available_reference():
        return None
    ref = Reference()
    ctx = ref.ctx(threads)
    t = ref.view(cfg.dtype, cfg.rows, cfg.cols, packed)
    xp = np.ascontiguousarray(WL.pad_cols(X[:1], cfg.cols)[0])
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
    o = Oracle()
    xp = WL.pad_cols(X[:1], cfg.cols)
    n, t0 = 0, time.perf_counter()
    while True:
        o.gemv(cfg.dtype, packed, cfg.rows, cfg.cols, xp, nthreads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s and n >= 2:
            break
    return el / n, n


def cpu_baseline(cfg, packed, X, budget_s=8.0):
    threads = os.cpu_count() or 1
    per_call_bytes = algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols, 1)
    r = None
    kind = "port"
    if cfg.dtype in (WL.DTYPE_Q4_0, WL.DTYPE_Q8_0):
        r = cpu_reference_time(cfg, packed, X, budget_s, threads)
        kind = "reference"
    if r is None:
        r = cpu_port_time(cfg, packed, X, budget_s, threads)
        kind = "port"
    sec, n = r
    return dict(host_cpu(), value=round(per_call_bytes / sec / 1e9, 3), unit=UNIT, cores=threads, kind=kind,
                sample=f"{n} full {cfg.rows}x{cfg.cols} GEMV calls (batch 1), {sec * 1e3:.2f} ms each, "
                       f"{'reference kernel_gemv thread pool' if kind == 'reference' else 'oracle C port (no reference ternary kernel)'} "
                       f"with {threads} threads")


# ----------------------------------------------------------- reference arm ---
def run_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.oracle import Oracle
    # Quantise with the oracle quantiser (same bytes as the GPU quantiser) so
    # this arm needs no GPU and no GPU library.
    src, X = WL.make_inputs(cfg, seed=0)
    o = Oracle()
    packed = o.pack_tq2(*src) if cfg.dtype == WL.DTYPE_TQ2_0 else o.quantize(cfg.dtype, src)
    del src
    threads = os.cpu_count() or 1
    bytes_per = algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols)
    ref_kernel = cfg.dtype in (WL.DTYPE_Q4_0, WL.DTYPE_Q8_0)
    fn = cpu_reference_time if ref_kernel else cpu_port_time
    kind = "reference" if ref_kernel else "port"
    for _ in range(args.warmup):
        fn(cfg, packed, X, 0.0, threads)
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
            "config": gemv_config(cfg, args.gpus),
            "execution": f"reference kernel_gemv thread pool on the host, {threads} threads (rank 0 only)"
                         if ref_kernel else f"oracle C port on the host, {threads} threads (rank 0 only)",
            "cpu_baseline": dict(host_cpu(), value=round(value, 3), unit=UNIT, cores=threads, kind=kind,
                                 sample=f"{args.steps} timed full GEMV calls after {args.warmup} warm-up"),
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- GPU env ----
class Env:
    """One process per GPU: torch device, optional NCCL process group, and
    the library context (sharded when world > 1)."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        import sapphire_b200 as sp
        self.torch, self.dist, self.sp = torch, dist, sp
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                    device_id=torch.device("cuda", self.local))
        self.ctx = sp.Context(num_threads=1, device=self.local)
        if self.world > 1:
            uid = torch.zeros(sp.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
            if self.rank == 0:
                uid.copy_(torch.frombuffer(bytearray(sp.shard_unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            self.ctx.shard(self.rank, self.world, bytes(uid.cpu().numpy().tobytes()))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, values):
        t = self.torch.tensor([float(v) for v in values], device="cuda", dtype=self.torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def all_true(self, flag: bool) -> bool:
        t = self.torch.tensor([0 if flag else 1], device="cuda", dtype=self.torch.int32)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return int(t.item()) == 0

    def ranks_identical(self, arr: np.ndarray) -> bool:
        """True when every rank holds the same bytes (sha256 compared)."""
        h = np.frombuffer(hashlib.sha256(np.ascontiguousarray(arr).tobytes()).digest()[:16], dtype=np.int64)
        mine = self.torch.from_numpy(h.copy()).cuda()
        if self.world == 1:
            return True
        allh = [self.torch.zeros_like(mine) for _ in range(self.world)]
        self.dist.all_gather(allh, mine)
        return all(self.torch.equal(allh[0], t) for t in allh)

    def sampler(self):
        return ClockSampler(self.local) if self.rank == 0 else NoSampler()

    def close(self):
        self.ctx.close()
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def build_weight(sp, ctx, cfg, seed=0):
    """Packed host bytes of the config's weight (GPU quantiser / packer) and x."""
    src, X = WL.make_inputs(cfg, seed=seed)
    if cfg.dtype == sp.DTYPE_TQ2_0:
        trits, scales = src
        packed = sp.pack_tq2(ctx, trits, scales)
    else:
        packed = sp.quantize(ctx, cfg.dtype, src)
    del src
    return packed, X


def elem_rel_err(y, ref, floor_frac=1e-3) -> float:
    """max_i |y_i - ref_i| / max(|ref_i|, floor_frac * max|ref|): per-element
    relative error with a floor (reported beside the normwise bar)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.maximum(np.abs(ref), floor_frac * max(float(np.max(np.abs(ref))), 1e-300))
    return float(np.max(np.abs(y - ref) / den))


def normwise(y, ref) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(y - ref)) / (den if den > 0 else 1.0))


def gemv_parity(env, cfg, y: np.ndarray, packed, X) -> dict:
    """Gathered y against the oracle (rank 0, f64 on the host) and across
    ranks (every rank's bytes hashed).  The oracle is the checker here, run
    after the timed region."""
    same = env.ranks_identical(y)
    out = {"ranks_identical": same, "checked": f"full y ({cfg.rows} rows) of one more product",
           "oracle": "oracle C restatement of the reference row kernels, f64"}
    ok = same
    if env.rank == 0:
        from oracle.oracle import Oracle
        ref = Oracle().gemv(cfg.dtype, packed, cfg.rows, cfg.cols, WL.pad_cols(X[:1], cfg.cols), f64=True,
                            nthreads=os.cpu_count() or 1)[0]
        err = normwise(y, ref)
        out.update({"normwise_err": float(f"{err:.3e}"), "elem_rel_err_floor1e-3": float(f"{elem_rel_err(y, ref):.3e}"),
                    "bar": GEMV_RTOL})
        ok = ok and err <= GEMV_RTOL and bool(np.isfinite(y).all())
    ok = env.all_true(ok)
    out["ok"] = ok
    return out


# ------------------------------------------------------------- GPU GEMV ------
def measure_gemv(args, env, cfg, with_cpu: bool) -> dict:
    torch, sp, ctx = env.torch, env.sp, env.ctx
    world, rank = env.world, env.rank
    # Two copies of the weight (different seeds) alternate between steps so
    # each step streams its weight from HBM.
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

    sampler = env.sampler()
    sampler.__enter__()
    for i in range(args.warmup):
        ctx.check(step(i), "warm-up")
    ctx.synchronize()

    # ---- device-timed region (value): K steps back to back on the lib stream
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    env.barrier()
    torch.cuda.synchronize()
    ctx.synchronize()
    # No event between steps: with programmatic dependent launch a step's
    # weight stream may start under the tail of the previous one, as in a
    # serving loop.
    t_all0.record(stream)
    for i in range(args.steps):
        ctx.check(step(i), "step")
    t_all1.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    sampler.__exit__()
    env.barrier()
    total_ms = t_all0.elapsed_time(t_all1)
    # Per-launch duration of one product alone (events around each launch).
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        ctx.check(step(i), "step")
        ends[i].record(stream)
    ctx.synchronize()
    kern_ms_local = float(np.mean([s.elapsed_time(e) for s, e in zip(starts, ends)]))
    total_ms, kern_ms = env.max_over_ranks([total_ms, kern_ms_local])
    ms_per_step = total_ms / args.steps
    value = bytes_per / (ms_per_step * 1e-3) / 1e9

    # ---- end-to-end through the public API with pinned host buffers
    x_host = torch.from_numpy(np.ascontiguousarray(X[:1])).pin_memory()
    y_host = torch.zeros((1, cfg.rows)).pin_memory()

    def e2e_step(i):
        return sp.lib.kernel_gemv(ctx.handle, y_host.data_ptr(), A[i & 1].handle, x_host.data_ptr())

    for i in range(args.warmup):
        ctx.check(e2e_step(i), "e2e warm-up")
    env.barrier()
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
    (e2e_ms,) = env.max_over_ranks([max(ev0.elapsed_time(ev1), wall * 1e3)])
    e2e_ms /= args.steps
    e2e_value = bytes_per / (e2e_ms * 1e-3) / 1e9

    # ---- parity of one more product (outside every timed region)
    y_dev.fill_(float("nan"))
    ctx.check(step(0), "parity product")
    ctx.synchronize()
    parity = gemv_parity(env, cfg, y_dev.cpu().numpy()[0], packed0, X)

    # ---- sharded: the rank's local slice as an unsharded GEMV on its own
    # context, timed the same way, so the gather's share of a step shows.
    breakdown = None
    if world > 1:
        row0, nloc = sp.shard_rows(cfg.rows, rank, world)
        rb = WL.row_bytes(cfg.dtype, cfg.cols)
        lctx = sp.Context(num_threads=1, device=env.local)
        AL = [sp.Tensor(cfg.dtype, (nloc, cfg.cols), pk[row0 * rb:(row0 + nloc) * rb]) for pk in (packed0, packed1)]
        for a in AL:
            lctx.check(sp.lib.kernel_tensor_upload(lctx.handle, a.handle), "upload slice")
        yl = torch.zeros(nloc, device="cuda")
        lstream = torch.cuda.ExternalStream(lctx.stream)

        def lstep(i):
            return sp.lib.kernel_gemv_device(lctx.handle, yl.data_ptr(), AL[i & 1].handle, x_dev.data_ptr())
        for i in range(args.warmup):
            lctx.check(lstep(i), "local warm-up")
        lctx.synchronize()
        l0 = torch.cuda.Event(enable_timing=True)
        l1 = torch.cuda.Event(enable_timing=True)
        l0.record(lstream)
        for i in range(args.steps):
            lctx.check(lstep(i), "local step")
        l1.record(lstream)
        lctx.synchronize()
        (local_ms,) = env.max_over_ranks([l0.elapsed_time(l1) / args.steps])
        for a in AL:
            a.release()
        lctx.close()
        breakdown = {"sharded_product_ms_per_step": round(ms_per_step, 5),
                     "local_gemv_ms_per_step": round(local_ms, 5),
                     "gather_and_sync_ms_per_step": round(ms_per_step - local_ms, 5),
                     "local_rows": nloc,
                     "how": "the rank's row slice timed as an unsharded GEMV (steps back to back, max over ranks); "
                            "the difference is the peer-memory gather and the wait for the slowest rank"}

    peaks = measured_peaks()
    per_rank_rows = (cfg.rows + world - 1) // world if world > 1 else cfg.rows
    kern_bytes = algorithmic_bytes(cfg.dtype, per_rank_rows, cfg.cols, 1)
    achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
    tag = f"gemv_{WL.DTYPE_NAMES[cfg.dtype].lower()}_{cfg.name}"
    gather = ("peer-memory gather fused into the GEMV: its epilogue stores 8-byte (epoch | value) words to every "
              "rank over NVLink and its warps then collect their slice of y")
    entry = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (PCG64 seed 0; N(0,0.02) weights quantised on the GPU, N(0,1) x)"
                if cfg.dtype != WL.DTYPE_TQ2_0 else
                "synthetic (PCG64 seed 0; trits uniform on {-1,0,1}, row scales U(0.01,0.1), N(0,1) x)",
        "config": gemv_config(cfg, world),
        "execution": f"row-shard x{world}, {gather}" if world > 1 else "pipelined GEMV kernel on one B200",
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "frac_sustained": round(kern_bytes / (ms_per_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                     "kernel_ms": round(kern_ms, 5), "traffic": ncu_traffic(tag), "kernel": tag,
                     "kernel_ms_covers": "one GEMV launch alone (events around it)" if world == 1
                     else "one sharded product alone: the GEMV with its fused peer-memory gather",
                     "frac_sustained_covers": "the same bytes over ms_per_step (steps back to back)"},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": 4 * cfg.cols,
                "d2h_bytes_per_step": 4 * cfg.rows, "ms_per_step": round(e2e_ms, 5),
                "path": "kernel_gemv with pinned host x/y (weights resident after upload): x copied in, "
                        "y written by the GEMV through the host mapping, then the stream synchronised"},
        "gpu_launches": args.steps,
        "parity": parity,
    }
    if breakdown:
        entry["breakdown"] = breakdown
    if rank == 0:
        entry["clocks"] = sampler.summary()
    if with_cpu and rank == 0:
        entry["cpu_baseline"] = cpu_baseline(cfg, packed0, X)
    for a in A:
        a.release()
    return entry


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
    xs = WL.pad_cols(bf16_round(X[:tokens]), cfg.cols)
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


def prefill_cpu_baseline(cfg, packed, X, budget_s=6.0):
    threads = os.cpu_count() or 1
    el, kind = cpu_prefill_time(cfg, packed, X, 4, threads)
    tokens = int(max(4, min(cfg.batch, 4 * budget_s / max(el, 1e-6))))
    el, kind = cpu_prefill_time(cfg, packed, X, tokens, threads)
    return dict(host_cpu(), value=round(prefill_flops(cfg, tokens) / el / 1e12, 5), unit=PREFILL_UNIT,
                cores=threads, kind=kind,
                sample=f"{tokens} of the {cfg.batch} tokens, one "
                       f"{'reference kernel_gemv' if kind == 'reference' else 'oracle port GEMV'}"
                       f" call per token ({el / tokens * 1e3:.2f} ms each) with {threads} threads")


def run_reference_prefill(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.oracle import Oracle
    src, X = WL.make_inputs(cfg, seed=0)
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
            "config": prefill_config(cfg, args.gpus),
            "execution": f"reference kernel_gemv per token on the host, {threads} threads (rank 0 only); "
                         f"each step {tokens} of the {cfg.batch} tokens",
            "cpu_baseline": dict(host_cpu(), value=round(value, 5), unit=PREFILL_UNIT, cores=threads, kind=kind,
                                 sample=f"each step {tokens} of the {cfg.batch} tokens, one kernel_gemv per token"),
            "e2e": {"value": round(value, 5), "unit": PREFILL_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def measure_prefill(args, env, cfg, with_cpu: bool) -> dict:
    torch, sp, ctx = env.torch, env.sp, env.ctx
    world, rank = env.world, env.rank
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

    sampler = env.sampler()
    sampler.__enter__()
    for i in range(args.warmup):
        ctx.check(step(i), "warm-up")
    ctx.synchronize()
    t0e = torch.cuda.Event(enable_timing=True)
    t1e = torch.cuda.Event(enable_timing=True)
    env.barrier()
    torch.cuda.synchronize()
    t0e.record(stream)
    for i in range(args.steps):
        ctx.check(step(i), "step")
    t1e.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    sampler.__exit__()
    env.barrier()
    (total_ms,) = env.max_over_ranks([t0e.elapsed_time(t1e)])
    ms_per_step = total_ms / args.steps
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
        del Xb

    # End to end through kernel_gemm with pinned host buffers (X in, Y out).
    xh = [torch.from_numpy(np.ascontiguousarray(X)).pin_memory(), torch.from_numpy(np.ascontiguousarray(X1)).pin_memory()]
    yh = torch.zeros((cfg.batch, cfg.rows)).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step(i):
        return sp.lib.kernel_gemm(ctx.handle, yh.data_ptr(), A[i & 1].handle, xh[i & 1].data_ptr(), cfg.batch,
                                  cfg.rows)
    for i in range(args.warmup):
        ctx.check(e2e_step(i), "e2e warm-up")
    env.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    w0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.check(e2e_step(i), "e2e step")
    ev1.record(stream)
    ctx.synchronize()
    (e2e_ms,) = env.max_over_ranks([max(ev0.elapsed_time(ev1), (time.perf_counter() - w0) * 1e3)])
    e2e_ms /= e2e_steps

    # ---- parity: one more product; 16 tokens spread over the batch against
    # the oracle on bf16-rounded activations, all of Y hashed across ranks.
    Yd.fill_(float("nan"))
    ctx.check(step(0), "parity product")
    ctx.synchronize()
    Y = Yd.cpu().numpy()
    same = env.ranks_identical(Y)
    parity = {"ranks_identical": same, "oracle": "oracle C restatement of the reference row kernels, f64, "
                                                  "on bf16-rounded activations"}
    ok = same and bool(np.isfinite(Y).all())
    if rank == 0:
        from oracle.oracle import Oracle
        idx = np.linspace(0, cfg.batch - 1, 16).astype(int)
        ref = Oracle().gemv(cfg.dtype, packed0, cfg.rows, cfg.cols, WL.pad_cols(bf16_round(X[idx]), cfg.cols),
                            f64=True, nthreads=os.cpu_count() or 1)
        err = normwise(Y[idx], ref)
        parity.update({"checked": f"{len(idx)} of {cfg.batch} token rows of Y (all {cfg.rows} columns); "
                                  f"all of Y for ranks_identical",
                       "normwise_err": float(f"{err:.3e}"), "bar": GEMV_RTOL})
        ok = ok and err <= GEMV_RTOL
    parity["ok"] = env.all_true(ok)

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
    entry = {
        "metric": PREFILL_METRIC, "value": round(value, 3), "unit": PREFILL_UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (PCG64 seed 0; N(0,0.02) weights quantised on the GPU, N(0,1) X)",
        "config": prefill_config(cfg, world),
        "execution": (f"row-shard x{world}: tcgen05 product per rank + NCCL all-gather" if world > 1
                      else "fp32->bf16 conversion + tcgen05 product on one B200"),
        "roofline": roof,
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": PREFILL_UNIT,
                "h2d_bytes_per_step": 4 * cfg.batch * cfg.cols, "d2h_bytes_per_step": 4 * cfg.batch * cfg.rows,
                "ms_per_step": round(e2e_ms, 4), "path": "kernel_gemm with pinned host X/Y"},
        "gpu_launches": 2 * args.steps,
        "parity": parity,
    }
    if rank == 0:
        entry["clocks"] = sampler.summary()
    if with_cpu and rank == 0:
        entry["cpu_baseline"] = prefill_cpu_baseline(cfg, packed0, X)
    for a in A:
        a.release()
    return entry


# -------------------------------------------------------------- decode -----
DECODE_METRIC = "Gemma-3-270M decode tok/s (greedy, Q4_0 projections and LM head)"
DECODE_UNIT = "tok/s"


def decode_bytes_per_token(cfg, pos: int) -> int:
    """Algorithmic HBM bytes of one generated token at position `pos`: every
    packed Q4_0 projection and the LM head, the embedding row, the KV rows the
    attention reads (the window for local layers) and writes, x/y vectors
    neglected (< 0.1 %)."""
    w = 0
    for _, rows, cols in cfg.projections():
        w += rows * WL.row_bytes(WL.DTYPE_Q4_0, cols)
    w *= cfg.layers
    w += cfg.vocab * WL.row_bytes(WL.DTYPE_Q4_0, cfg.hidden) + 2 * cfg.hidden
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
    return dict(host_cpu(), value=round(n / td, 3), unit=DECODE_UNIT, cores=os.cpu_count() or 1, kind="reference",
                sample=f"one reference decode (its inference_forward per token, Q4_0 kernel_gemv, all host "
                       f"threads): {cfg.prompt}-token prompt in {tp:.1f} s, then {n} greedy tokens in {td:.2f} s")


def run_reference_decode(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.oracle import Oracle, available_reference_decode
    if not available_reference_decode():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdecode_ref.so not built "
                          "(make -C oracle ref needs the reference sources)"}), flush=True)
        return 0
    o = Oracle()
    model = WL.make_decode_model(cfg, lambda a: o.quantize(3, a), seed=0)
    n_gen = max(1, min(args.steps, cfg.generate))
    cb = decode_cpu_baseline(cfg, model, n_gen=n_gen)
    line = {"impl": "reference", "metric": DECODE_METRIC, "value": cb["value"], "unit": DECODE_UNIT,
            "n_gpus": args.gpus, "steps": n_gen, "warmup": 0, "ms_per_step": round(1e3 / cb["value"], 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (PCG64 seed 0, random-init Gemma-3-270M)",
            "config": decode_config(cfg, args.gpus),
            "execution": "reference inference_forward per token on the host thread pool (rank 0 only); "
                         "a step is one generated token",
            "cpu_baseline": dict(cb, sample=cb["sample"] + "; a step is one generated token"),
            "e2e": {"value": cb["value"], "unit": DECODE_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def measure_decode(args, env, cfg, with_cpu: bool, steps: int, warmup: int) -> dict:
    """Each step is one full request: the 512-token prompt, then 64 greedy
    tokens.  `value` is generated tokens per second of the generation phase
    (device events).  N > 1 serves the same request on every rank with the
    LM head row-sharded: each rank computes its slice of the logits and the
    ranks exchange 8-byte (value, index) words to agree on the token."""
    torch, sp, ctx = env.torch, env.sp, env.ctx
    from sapphire_b200.decode import Decoder
    world, rank = env.world, env.rank
    model = WL.make_decode_model(cfg, lambda a: sp.quantize(ctx, 3, a), seed=0)
    dctx = ctx
    dec = Decoder(dctx, cfg, model)
    prompt = model["prompt"]
    sampler = env.sampler()
    sampler.__enter__()
    for _ in range(warmup):
        dec.generate(prompt, cfg.generate)
    env.barrier()
    torch.cuda.synchronize()
    gen_ms, prompt_ms, walls = [], [], []
    ids = None
    for _ in range(steps):
        w0 = time.perf_counter()
        ids, _ = dec.generate(prompt, cfg.generate)
        walls.append(time.perf_counter() - w0)
        pm, gm = dec.last_times()
        prompt_ms.append(pm)
        gen_ms.append(gm)
    torch.cuda.synchronize()
    sampler.__exit__()
    gen_total, prompt_total, wall_total = env.max_over_ranks(
        [float(np.sum(gen_ms)), float(np.sum(prompt_ms)), float(np.sum(walls))])
    n_tok = cfg.generate * steps
    value = n_tok / (gen_total * 1e-3)
    golden = os.path.join(ROOT, "tests", "golden", "decode_gemma3_270m_seed0.npz")
    match = bool(np.array_equal(ids, np.load(golden)["tokens"])) if os.path.exists(golden) else False
    all_match = env.all_true(match)
    peaks = measured_peaks()
    bpt = float(np.mean([decode_bytes_per_token(cfg, cfg.prompt - 1 + g) for g in range(cfg.generate)]))
    ms_tok = gen_total / n_tok
    exec_kind = ("one persistent kernel for all layers, then the LM head and the argmax"
                 if dec.launches_per_prompt_token == 1 else "one kernel per stage")
    achieved = bpt / (ms_tok * 1e-3) / 1e9
    entry = {
        "metric": DECODE_METRIC, "value": round(value, 2), "unit": DECODE_UNIT, "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(gen_total / steps, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (PCG64 seed 0; random-init Gemma-3-270M, N(0,0.02) weights, Q4_0 projections "
                "and LM head, bf16 embedding, zero norm weights)",
        "config": decode_config(cfg, world),
        "execution": (f"device-resident decode step in CUDA graphs ({exec_kind})" if world == 1 else
                      f"device-resident decode step in CUDA graphs ({exec_kind}) on every rank, LM-head rows "
                      "sharded, argmax agreed through 8-byte peer-memory words"),
        "prompt_tok_s": round((cfg.prompt - 1) * steps / (prompt_total * 1e-3), 1),
        "tokens_match_reference": all_match,
        "parity": {"ok": all_match, "checked": f"all {cfg.generate} greedy ids of every rank against the "
                                              "reference decode's golden ids"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "kernel_ms": round(ms_tok, 5), "traffic": None,
                     "kernel": "decode step graph (generation phase, per token)", "bytes_per_token": int(bpt)},
        "e2e": {"value": round(n_tok / wall_total, 2), "unit": DECODE_UNIT,
                "h2d_bytes_per_step": 4 * cfg.prompt, "d2h_bytes_per_step": 8 * cfg.generate,
                "ms_per_step": round(wall_total / steps * 1e3, 3),
                "path": "sapphire_decoder_generate with a host prompt and host ids (prompt phase included)"},
        "gpu_launches": steps * (cfg.generate * dec.launches_per_token
                                 + (cfg.prompt - 1) * dec.launches_per_prompt_token),
    }
    if rank == 0:
        entry["clocks"] = sampler.summary()
    if with_cpu and rank == 0:
        cb = decode_cpu_baseline(cfg, model)
        if cb:
            entry["cpu_baseline"] = cb
    dec.close()
    return entry


# ----------------------------------------------------------------- main -----
def run_gpu(args, cfg) -> int:
    env = Env()
    with_cpu = env.world == 1 and not args.no_cpu_baseline
    if cfg is WL.C3:
        line = measure_decode(args, env, cfg, with_cpu, args.steps, args.warmup)
    elif cfg.batch > 1:
        line = measure_prefill(args, env, cfg, with_cpu)
    else:
        line = measure_gemv(args, env, cfg, with_cpu)
    if args.secondary:
        sec = {}
        for c in (WL.C2_Q4, WL.C2_TQ2, WL.C4):
            sec[c.name] = measure_gemv(args, env, c, with_cpu)
        sec[WL.C5.name] = measure_prefill(args, env, WL.C5, with_cpu)
        # Decode: a step is a whole request (~0.5 s); a few are enough.
        sec[WL.C3.name] = measure_decode(args, env, WL.C3, with_cpu, steps=min(args.steps, 3), warmup=1)
        line["secondary"] = sec
    ok = line["parity"]["ok"] and all(e["parity"]["ok"] for e in line.get("secondary", {}).values())
    env.close()
    if env.rank == 0:
        print(json.dumps(line), flush=True)
    return 0 if ok else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="sapphire", choices=["sapphire", "reference"])
    ap.add_argument("--config", default=None,
                    help="one configuration only (default: the Q8_0 LM head with every other "
                         "configuration in `secondary`)")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    name = args.config or WL.C2.name
    args.secondary = args.config is None and not args.no_secondary and args.impl != "reference"
    cfg = WL.C3 if name == WL.C3.name else WL.CONFIGS[name]
    if args.impl == "reference":
        if cfg is WL.C3:
            return run_reference_decode(args, cfg)
        if cfg.batch > 1:
            return run_reference_prefill(args, cfg)
        return run_reference_arm(args, cfg)
    return run_gpu(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
