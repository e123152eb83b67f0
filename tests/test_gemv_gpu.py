"""GPU parity of the B200 GEMV path against the oracle and the reference's
golden outputs, through the C-ABI (libsapphire_cuda.so).

Bars: packing / unpacking bit-exact; GEMV normwise relative error
max|y - y_ref| / max|y_ref| <= 1e-4 (GEMV_RTOL) against the fp32 reference.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import GEMV_RTOL, normwise_rel
from oracle.oracle import Q4_0, Q8_0, TQ2_0, F32, BF16
from sapphire_b200 import workloads

pytestmark = pytest.mark.gpu


def rand_packed(oracle, dtype, rows, cols, seed):
    rng = np.random.default_rng(seed)
    if dtype == TQ2_0:
        trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
        scales = rng.uniform(0.01, 0.1, size=rows).astype(np.float32)
        return oracle.pack_tq2(trits, scales)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    if dtype == F32:
        return w.reshape(-1).view(np.uint8).copy()
    if dtype == BF16:
        return (w.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).copy()
    return oracle.quantize(dtype, w)


def oracle_y(oracle, dtype, packed, rows, cols, X):
    return oracle.gemv(dtype, packed, rows, cols, workloads.pad_cols(np.atleast_2d(X), cols), f64=True)


# ------------------------------------------------------------- packing -----
@pytest.mark.parametrize("dtype", [Q4_0, Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 32), (3, 70), (64, 640), (2048, 640)])
def test_quantizer_bit_exact(sp, ctx, oracle, dtype, rows, cols):
    rng = np.random.default_rng(rows + cols + dtype)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    w[0, :5] = [0.0, -0.0, 1e-30, -3.0, 3.0]       # ties and tiny values
    if rows > 1:
        w[1, :] = 0.0                                # all-zero row
    gpu = sp.quantize(ctx, dtype, w)
    assert np.array_equal(gpu, oracle.quantize(dtype, w))


def test_quantizer_seeded_c1_digest(sp, ctx, oracle, seeded):
    import hashlib
    w, _ = workloads.make_inputs(workloads.C1, seed=0)
    gpu = sp.quantize(ctx, Q4_0, w)
    assert hashlib.sha256(gpu.tobytes()).hexdigest() == str(seeded["c1_packed_sha256"])


@pytest.mark.parametrize("rows,cols", [(1, 32), (5, 100), (512, 1000)])
def test_ternary_pack_bit_exact(sp, ctx, oracle, rows, cols):
    rng = np.random.default_rng(rows * cols)
    trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
    scales = rng.uniform(0.01, 0.1, size=rows).astype(np.float32)
    assert np.array_equal(sp.pack_tq2(ctx, trits, scales), oracle.pack_tq2(trits, scales))


def test_ternary_pack_rejects_bad_trits(sp, ctx):
    trits = np.zeros((2, 32), dtype=np.int8)
    trits[1, 7] = 2
    with pytest.raises(sp.SapphireError):
        sp.pack_tq2(ctx, trits, np.ones(2, dtype=np.float32))


@pytest.mark.parametrize("dtype", [Q4_0, Q8_0, TQ2_0, F32, BF16])
def test_unpack_bit_exact(sp, ctx, oracle, dtype):
    rows, cols = 37, 100
    packed = rand_packed(oracle, dtype, rows, cols, seed=11)
    A = sp.Tensor(dtype, (rows, cols), packed)
    assert np.array_equal(sp.dequantize(ctx, A), oracle.dequantize(dtype, packed, rows, cols))


# ------------------------------------------------- reference golden outputs -
def test_dispatch_pattern(sp, ctx, patterns):
    row, x = patterns["dispatch_row"], patterns["dispatch_x"]
    A = sp.Tensor(Q4_0, (1, 128), row)
    y = sp.gemv(ctx, A, x)
    assert abs(y[0] - float(patterns["dispatch_aligned"])) < 1e-4   # test_dispatch.c:37


@pytest.mark.parametrize("tag,dtype", [("bq4", Q4_0), ("bq8", Q8_0)])
def test_bench_patterns(sp, ctx, patterns, tag, dtype):
    rows, cols = (int(v) for v in patterns[f"{tag}_shape"])
    A = sp.Tensor(dtype, (rows, cols), patterns[f"{tag}_W"])
    y = sp.gemv(ctx, A, patterns[f"{tag}_x"])
    assert normwise_rel(y, patterns[f"{tag}_y"]) < GEMV_RTOL


@pytest.mark.parametrize("i", range(5))
def test_end_to_end_patterns(sp, ctx, patterns, i):
    import sys
    from conftest import GOLDEN
    sys.path.insert(0, GOLDEN)
    import make_golden
    rows, cols = (int(v) for v in patterns[f"e2e_{i}_shape"])
    if f"e2eq4_{i}_W" in patterns:
        q4, q8 = patterns[f"e2eq4_{i}_W"], patterns[f"e2eq8_{i}_W"]
        x = (np.float32(0.001) * np.arange(1, cols + 1, dtype=np.float32)).astype(np.float32)
    else:
        q4, q8, x = make_golden.pattern_e2e(rows, cols // 32)
    for dt, W, key in ((Q4_0, q4, "q4"), (Q8_0, q8, "q8")):
        y = sp.gemv(ctx, sp.Tensor(dt, (rows, cols), W), x)
        assert normwise_rel(y, patterns[f"e2e{key}_{i}_y"]) < GEMV_RTOL
        assert abs(y.astype(np.float64).sum() - float(patterns[f"e2e{key}_{i}_sum"])) <= \
            1e-4 * max(1.0, abs(float(patterns[f"e2e{key}_{i}_sum"])))


SEEDED = [("c1", workloads.C1),
          ("q8_small", workloads.GemvConfig("q8_0_4096x640", Q8_0, 4096, 640)),
          ("q4_ragged", workloads.GemvConfig("q4_0_100x80", Q4_0, 100, 80)),
          ("q8_ragged", workloads.GemvConfig("q8_0_33x70", Q8_0, 33, 70)),
          ("q4_prefill_rows", workloads.GemvConfig("q4_0_256x2560", Q4_0, 256, 2560, batch=4))]


@pytest.mark.parametrize("tag,cfg", SEEDED, ids=[t for t, _ in SEEDED])
def test_seeded_against_reference_outputs(sp, ctx, seeded, tag, cfg):
    w, X = workloads.make_inputs(cfg, seed=0)
    packed = sp.quantize(ctx, cfg.dtype, w)          # product quantiser
    A = sp.Tensor(cfg.dtype, (cfg.rows, cfg.cols), packed)
    Y = sp.gemm(ctx, A, np.ascontiguousarray(X), cfg.batch)
    assert normwise_rel(Y, seeded[f"{tag}_Y"]) < GEMV_RTOL


def test_ternary_seeded_fixture(sp, ctx, seeded):
    cfg = workloads.GemvConfig("tq2_0_512x1000", TQ2_0, 512, 1000)
    (trits, scales), X = workloads.make_inputs(cfg, seed=0)
    packed = sp.pack_tq2(ctx, trits, scales)
    y = sp.gemv(ctx, sp.Tensor(TQ2_0, (cfg.rows, cfg.cols), packed), X[0])
    assert normwise_rel(y, seeded["tq2_Y_oracle_f64"][0]) < GEMV_RTOL


# ---------------------------------------------------------- shape sweep ----
SHAPES = [(1, 32), (1, 1), (31, 32), (33, 64), (100, 80), (257, 96), (2048, 640), (640, 2048),
          (1000, 2560), (64, 16384)]


@pytest.mark.parametrize("dtype", [Q4_0, Q8_0, TQ2_0, F32, BF16])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_shapes(sp, ctx, oracle, dtype, rows, cols):
    packed = rand_packed(oracle, dtype, rows, cols, seed=rows * 7 + cols)
    x = np.random.default_rng(cols).standard_normal(cols, dtype=np.float32)
    y = sp.gemv(ctx, sp.Tensor(dtype, (rows, cols), packed), x)
    assert normwise_rel(y, oracle_y(oracle, dtype, packed, rows, cols, x)[0]) < GEMV_RTOL


SPLIT_SHAPES = [(Q8_0, 4096, 640), (Q4_0, 4096, 2560), (TQ2_0, 64, 16384), (TQ2_0, 2048, 4096),
                (Q4_0, 33, 16384), (F32, 100, 3000), (BF16, 700, 4100)]


def test_pipelined_split_tiles_deterministic_and_repeatable(sp, ctx, oracle):
    # Shapes whose 32-row tiles are shared by several warps of the persistent
    # kernel: the combine must be exact to the oracle bar, bitwise repeatable,
    # and leave its counters at zero for the next call (interleaved shapes).
    cases = []
    for dtype, rows, cols in SPLIT_SHAPES:
        packed = rand_packed(oracle, dtype, rows, cols, seed=rows + cols)
        x = np.random.default_rng(rows).standard_normal(cols, dtype=np.float32)
        A = sp.Tensor(dtype, (rows, cols), packed)
        cases.append((A, x, oracle_y(oracle, dtype, packed, rows, cols, x)[0]))
    first = [sp.gemv(ctx, A, x) for A, x, _ in cases]
    for _ in range(3):
        for (A, x, ref), y0 in zip(cases, first):
            y = sp.gemv(ctx, A, x)
            assert np.array_equal(y, y0)
            assert normwise_rel(y, ref) < GEMV_RTOL


@pytest.mark.parametrize("dtype", [Q4_0, Q8_0, TQ2_0, F32])
@pytest.mark.parametrize("batch", [2, 3, 8, 11])
def test_gemm_batched(sp, ctx, oracle, dtype, batch):
    rows, cols = 300, 640
    packed = rand_packed(oracle, dtype, rows, cols, seed=batch)
    X = np.random.default_rng(batch).standard_normal((batch, cols), dtype=np.float32)
    A = sp.Tensor(dtype, (rows, cols), packed)
    Y = sp.gemm(ctx, A, X, batch)
    assert normwise_rel(Y, oracle_y(oracle, dtype, packed, rows, cols, X)) < GEMV_RTOL
    # out_stride == 0 takes the single-vector path (reference dispatch.c:98)
    Y0 = np.full((batch, rows), 7.0, dtype=np.float32)
    sp.gemm(ctx, A, X, batch, Y=Y0, out_stride=0)
    assert normwise_rel(Y0[0], Y[0]) < 1e-6 and (Y0[1:] == 7.0).all()


def test_unaligned_x_pointer(sp, ctx, oracle):
    rows, cols = 128, 256
    packed = rand_packed(oracle, Q4_0, rows, cols, seed=5)
    buf = np.random.default_rng(5).standard_normal(cols + 1, dtype=np.float32)
    xaddr = buf.ctypes.data + 4                     # bench_q4's x + 1
    y = np.zeros(rows, dtype=np.float32)
    A = sp.Tensor(Q4_0, (rows, cols), packed)
    assert sp.lib.kernel_gemv(ctx.handle, y.ctypes.data, A.handle, xaddr) == 0
    assert normwise_rel(y, oracle_y(oracle, Q4_0, packed, rows, cols, buf[1:])[0]) < GEMV_RTOL


@pytest.mark.parametrize("dtype,rows,cols", [(Q8_0, 262144, 640), (Q4_0, 4096, 640), (TQ2_0, 1000, 16384),
                                            (Q4_0, 2048, 640), (F32, 300, 96)])
def test_page_locked_host_y(sp, ctx, oracle, dtype, rows, cols):
    """kernel_gemv into page-locked host y: the kernel writes the rows through
    the host mapping (no copy after the product); the result is bit for bit
    the one of the copy path (pageable y) and within the bar of the oracle."""
    packed = rand_packed(oracle, dtype, rows, cols, seed=21)
    A = sp.Tensor(dtype, (rows, cols), packed)
    x = np.random.default_rng(21).standard_normal(cols, dtype=np.float32)
    y_copy = np.zeros(rows, dtype=np.float32)
    assert sp.lib.kernel_gemv(ctx.handle, y_copy.ctypes.data, A.handle, x.ctypes.data) == 0
    hp = sp.lib.kernel_host_alloc(rows * 4)
    assert hp
    try:
        y_pin = np.ctypeslib.as_array(C.cast(hp, C.POINTER(C.c_float)), shape=(rows,))
        for _ in range(2):
            y_pin[:] = np.nan
            assert sp.lib.kernel_gemv(ctx.handle, hp, A.handle, x.ctypes.data) == 0
            assert np.array_equal(y_pin, y_copy)
        assert normwise_rel(y_pin, oracle_y(oracle, dtype, packed, rows, cols, x)[0]) < GEMV_RTOL
    finally:
        sp.lib.kernel_host_free(hp)


def test_device_pointer_path(sp, ctx, oracle):
    import torch
    rows, cols = 4096, 640
    packed = rand_packed(oracle, Q8_0, rows, cols, seed=9)
    A = sp.Tensor(Q8_0, (rows, cols), packed)
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    assert sp.lib.kernel_gemv_device(ctx.handle, y.data_ptr(), A.handle, x.data_ptr()) == 0
    ctx.synchronize()
    ref = oracle_y(oracle, Q8_0, packed, rows, cols, x.cpu().numpy())[0]
    assert normwise_rel(y.cpu().numpy(), ref) < GEMV_RTOL
    # the same device buffers through the synchronous entry point
    y2 = torch.zeros(rows, device="cuda")
    assert sp.lib.kernel_gemv(ctx.handle, y2.data_ptr(), A.handle, x.data_ptr()) == 0
    assert torch.equal(y, y2)
    # device-resident weights (AoS bytes already on the GPU)
    wd = torch.from_numpy(packed).cuda()
    Ad = sp.Tensor(Q8_0, (rows, cols), wd)
    y3 = torch.zeros(rows, device="cuda")
    assert sp.lib.kernel_gemv(ctx.handle, y3.data_ptr(), Ad.handle, x.data_ptr()) == 0
    assert torch.equal(y, y3)


def test_weight_cache_lifecycle(sp, ctx, oracle):
    rows, cols = 256, 640
    packed = rand_packed(oracle, Q4_0, rows, cols, seed=1)
    A = sp.Tensor(Q4_0, (rows, cols), packed)
    before = ctx.resident_bytes()
    assert sp.lib.kernel_tensor_upload(ctx.handle, A.handle) == 0
    assert ctx.resident_bytes() == before + rows * 640 // 32 * 20
    assert sp.lib.kernel_tensor_upload(ctx.handle, A.handle) == 0          # idempotent
    assert ctx.resident_bytes() == before + rows * 640 // 32 * 20
    x = np.ones(cols, dtype=np.float32)
    y1 = sp.gemv(ctx, A, x)
    assert sp.lib.kernel_tensor_evict(ctx.handle, A.handle) == 0
    assert ctx.resident_bytes() == before
    # new host bytes after an explicit evict are picked up
    packed2 = rand_packed(oracle, Q4_0, rows, cols, seed=2)
    packed[:] = packed2
    y2 = sp.gemv(ctx, A, x)
    assert not np.array_equal(y1, y2)
    assert normwise_rel(y2, oracle_y(oracle, Q4_0, packed2, rows, cols, x)[0]) < GEMV_RTOL
    A.release()                                                        # release drops the copy
    assert ctx.resident_bytes() == before


# ------------------------------------------- reference test_tensor_gemv.c ---
def fview(sp, m, n, vals):
    return sp.Tensor(F32, (m, n), np.asarray(vals, dtype=np.float32).reshape(m, n).copy())


def test_dense_basic_and_null_context(sp, ctx):
    A = fview(sp, 3, 4, range(1, 13))
    x = np.ones(4, dtype=np.float32)
    assert np.allclose(sp.gemv(ctx, A, x), [10, 26, 42], atol=1e-5)       # test_tensor_gemv.c:52-54
    assert np.allclose(sp.gemv(None, A, x), [10, 26, 42], atol=1e-5)      # NULL ctx works for F32


def test_dense_gemv_add(sp, ctx):
    A = fview(sp, 3, 2, [1, 0, 0, 1, 1, 1])
    x = np.array([2, 3], dtype=np.float32)
    y = np.array([10, 20, 30], dtype=np.float32)
    assert sp.lib.kernel_gemv_add(ctx.handle, y.ctypes.data, A.handle, x.ctypes.data, 1.0) == 0
    assert np.allclose(y, [12, 23, 35], atol=1e-5)                        # test_tensor_gemv.c:193-195
    B = fview(sp, 2, 2, [1, 1, 1, 1])
    y = np.zeros(2, dtype=np.float32)
    x = np.array([2, 2], dtype=np.float32)
    assert sp.lib.kernel_gemv_add(ctx.handle, y.ctypes.data, B.handle, x.ctypes.data, 0.5) == 0
    assert np.allclose(y, [2, 2], atol=1e-5)


def test_dense_gemv_batch_and_tensor(sp, ctx):
    A = fview(sp, 2, 2, [1, 2, 3, 4])
    X = np.array([1, 0, 0, 1, 1, 1], dtype=np.float32)
    Y = np.zeros(6, dtype=np.float32)
    assert sp.lib.kernel_gemv_batch(ctx.handle, Y.ctypes.data, A.handle, X.ctypes.data, 3) == 0
    assert np.allclose(Y, [1, 3, 2, 4, 3, 7], atol=1e-5)                  # test_tensor_gemv.c:275-277
    L = sp.lib
    yt = L.tensor_create(1, (C.c_int * 1)(4), F32)
    xt = L.tensor_create(1, (C.c_int * 1)(5), F32)
    At = L.tensor_create(2, (C.c_int * 2)(4, 5), F32)
    for i in range(20):
        L.tensor_set_f32(At, i, 2.0)
    for i in range(5):
        L.tensor_set_f32(xt, i, 1.0)
    assert L.kernel_gemv_tensor(ctx.handle, yt, At, xt) == 0
    assert all(abs(L.tensor_get_f32(yt, i) - 10.0) < 1e-5 for i in range(4))
    for h in (yt, xt, At):
        L.tensor_release(h)


def test_dense_large(sp, ctx):
    A = sp.Tensor(F32, (256, 512), np.full(256 * 512, 0.01, dtype=np.float32))
    y = sp.gemv(ctx, A, np.ones(512, dtype=np.float32))
    assert np.abs(y - 5.12).max() < 0.01                                  # test_tensor_gemv.c:371-373


def test_uninitialized_context_rejected(sp):
    L = sp.lib
    c = L.kernel_ctx_create(1, 16)
    A = fview(sp, 2, 2, [1, 2, 3, 4])
    y = np.zeros(2, dtype=np.float32)
    x = np.ones(2, dtype=np.float32)
    assert L.kernel_gemv(c, y.ctypes.data, A.handle, x.ctypes.data) == -1  # pool.c:276-279
    assert L.kernel_ctx_init(c) == 0 and L.kernel_ctx_init(c) == 0        # idempotent
    assert L.kernel_gemv(c, y.ctypes.data, A.handle, x.ctypes.data) == 0
    L.kernel_ctx_destroy(c)


# ------------------------------------------------------------ row ABI -----
def test_row_abi(sp, patterns, oracle):
    row, x = patterns["dispatch_row"], patterns["dispatch_x"]
    for fn in (sp.lib.quantized_gemv_q4_0_aligned, sp.lib.quantized_gemv_q4_0_unaligned):
        assert abs(fn(row.ctypes.data, x.ctypes.data, 4, 32) - float(patterns["dispatch_aligned"])) < 1e-4
        assert fn(row.ctypes.data, x.ctypes.data, 4, 16) == 0.0                 # block_size != 32
    W, xq = patterns["bq8_W"], patterns["bq8_x"]
    v = sp.lib.quantized_gemv_q8_0_aligned(W.ctypes.data, xq.ctypes.data, 8, 32)
    assert abs(v - float(patterns["bq8_y"][0])) <= 1e-4 * max(1, abs(float(patterns["bq8_y"][0])))
    packed = rand_packed(oracle, TQ2_0, 1, 96, seed=3)
    xt = np.random.default_rng(3).standard_normal(96, dtype=np.float32)
    v = sp.lib.quantized_gemv_tq2_0(packed.ctypes.data, xt.ctypes.data, 3, 32)
    assert abs(v - oracle_y(oracle, TQ2_0, packed, 1, 96, xt)[0, 0]) < 1e-4
    w = np.arange(8, dtype=np.float32)
    assert abs(sp.lib.quantized_gemv_f32_avx2(w.ctypes.data, np.ones(8, np.float32).ctypes.data, 8, 1) - 28) < 1e-5
    args = sp.GemmArgs(w.ctypes.data, np.ones(16, np.float32).ctypes.data, 0, 2, 8, 1, 8, 1)
    out = np.zeros(2, dtype=np.float32)
    args.Y = out.ctypes.data
    sp.lib.kernel_gemm_f32_avx2(C.byref(args))
    assert np.allclose(out, [28, 28])


# --------------------------------------------------- full-size properties --
def test_lm_head_full_size_q8_0(sp, ctx, oracle):
    cfg = workloads.C2
    w, X = workloads.make_inputs(cfg, seed=0)
    packed = sp.quantize(ctx, Q8_0, w)
    del w
    A = sp.Tensor(Q8_0, (cfg.rows, cfg.cols), packed)
    y = sp.gemv(ctx, A, X[0])
    ref = oracle.gemv(Q8_0, packed, cfg.rows, cfg.cols, X)[0]   # reference scalar order, fp32
    assert normwise_rel(y, ref) < GEMV_RTOL
    # linearity: A(a x1 + b x2) = a A x1 + b A x2 (size-independent property)
    x2 = np.random.default_rng(1).standard_normal(cfg.cols, dtype=np.float32)
    y2 = sp.gemv(ctx, A, x2)
    y12 = sp.gemv(ctx, A, (np.float32(0.5) * X[0] + np.float32(2.0) * x2).astype(np.float32))
    assert normwise_rel(y12, 0.5 * y.astype(np.float64) + 2.0 * y2) < GEMV_RTOL
    sp.lib.kernel_tensor_evict(ctx.handle, A.handle)


def test_ternary_full_size(sp, ctx, oracle):
    cfg = workloads.C4
    (trits, scales), X = workloads.make_inputs(cfg, seed=0)
    packed = sp.pack_tq2(ctx, trits, scales)
    del trits
    A = sp.Tensor(TQ2_0, (cfg.rows, cfg.cols), packed)
    y = sp.gemv(ctx, A, X[0])
    ref = oracle.gemv(TQ2_0, packed, cfg.rows, cfg.cols, X)[0]
    assert normwise_rel(y, ref) < GEMV_RTOL
    sp.lib.kernel_tensor_evict(ctx.handle, A.handle)


# ----------------------------------------- streaming kernel, odd geometry --
# Q8_0 / Q4_0 weights of more than 512 tiles or more than 64 blocks per row
# run the streaming kernel (smaller ones the latency-bound direct kernel);
# TQ2_0 always does.  Odd block counts leave the last 64-column unit with one
# block; ragged rows leave a partial last tile.
STREAM_SHAPES = [(Q8_0, 20000, 96), (Q8_0, 1000, 2080), (Q4_0, 16421, 96), (Q4_0, 777, 2080),
                 (Q4_0, 17000, 640), (TQ2_0, 100, 80), (TQ2_0, 3001, 2080), (TQ2_0, 33, 16384)]


@pytest.mark.parametrize("dtype,rows,cols", STREAM_SHAPES)
def test_stream_kernel_shapes(sp, ctx, oracle, dtype, rows, cols):
    packed = rand_packed(oracle, dtype, rows, cols, seed=rows + 3 * cols)
    x = np.random.default_rng(rows).standard_normal(cols, dtype=np.float32)
    A = sp.Tensor(dtype, (rows, cols), packed)
    y = sp.gemv(ctx, A, x)
    assert normwise_rel(y, oracle_y(oracle, dtype, packed, rows, cols, x)[0]) < GEMV_RTOL
    assert np.array_equal(y, sp.gemv(ctx, A, x))          # repeatable bit for bit


# ------------------------------------------- high-dynamic-range activations --
# x is converted to a 22-bit fixed-point image with one exponent for all of x
# (the streaming kernel and the Q8_0 direct kernel; the Q4_0 direct kernel
# uses fp32 x).  These cases stress that conversion: outliers 1e3 / 1e4 above
# the bulk, magnitudes spread over eight decades, an all-zero block beside a
# block of tiny values.  Bar: normwise error <= 1e-4 against the oracle in f64
# (the GEMV parity bar); the per-element relative error with a floor of
# 1e-3 * max|y| is printed and checked against a looser 5e-2 (a 1e4 outlier
# over 16384 N(0,1) columns puts the fixed-point step at 2^-8, about 1e-1 of
# accumulated error on a row, the size of an fp32 sum's own rounding there).
def hdr_x(kind: str, cols: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "outliers":
        x = rng.standard_normal(cols).astype(np.float32)
        i = rng.choice(cols, size=2, replace=False)
        x[i[0]] = np.float32(1e3) * rng.choice([-1, 1])
        x[i[1]] = np.float32(1e4) * rng.choice([-1, 1])
    elif kind == "decades":
        x = (10.0 ** rng.uniform(-6, 2, cols) * rng.choice([-1.0, 1.0], cols)).astype(np.float32)
    else:                                            # zero block and tiny block
        x = rng.standard_normal(cols).astype(np.float32)
        nb = cols // 32
        x[32 * (nb // 3): 32 * (nb // 3) + 32] = 0.0
        x[32 * (2 * nb // 3): 32 * (2 * nb // 3) + 32] *= np.float32(1e-7)
    return x


HDR_SHAPES = [(Q8_0, 20000, 640), (Q4_0, 20000, 640), (TQ2_0, 20000, 640), (Q8_0, 2048, 640),
              (Q4_0, 2048, 640), (Q8_0, 1024, 16384), (Q4_0, 1024, 16384), (TQ2_0, 1024, 16384)]


@pytest.mark.parametrize("kind", ["outliers", "decades", "zero_tiny"])
@pytest.mark.parametrize("dtype,rows,cols", HDR_SHAPES)
def test_high_dynamic_range_x(sp, ctx, oracle, dtype, rows, cols, kind):
    from conftest import elem_rel_floor
    packed = rand_packed(oracle, dtype, rows, cols, seed=rows + cols + dtype)
    x = hdr_x(kind, cols, seed=cols + dtype)
    y = sp.gemv(ctx, sp.Tensor(dtype, (rows, cols), packed), x)
    ref = oracle_y(oracle, dtype, packed, rows, cols, x)[0]
    nw, el = normwise_rel(y, ref), elem_rel_floor(y, ref)
    print(f"HDR {kind} dtype={dtype} {rows}x{cols}: normwise {nw:.3e} per-element(floor 1e-3) {el:.3e}")
    assert nw < GEMV_RTOL
    assert el < 5e-2


# --------------------------------------------- LM-head shape, all formats --
@pytest.mark.parametrize("cfg", [workloads.C2_Q4, workloads.C2_TQ2], ids=lambda c: c.name)
def test_lm_head_shape_q4_0_and_ternary(sp, ctx, oracle, cfg):
    src, X = workloads.make_inputs(cfg, seed=0)
    packed = sp.pack_tq2(ctx, *src) if cfg.dtype == TQ2_0 else sp.quantize(ctx, cfg.dtype, src)
    del src
    A = sp.Tensor(cfg.dtype, (cfg.rows, cfg.cols), packed)
    y = sp.gemv(ctx, A, X[0])
    ref = oracle.gemv(cfg.dtype, packed, cfg.rows, cfg.cols, X, f64=True)[0]
    assert normwise_rel(y, ref) < GEMV_RTOL
    sp.lib.kernel_tensor_evict(ctx.handle, A.handle)
