"""Pins the CPU oracle to the reference (CPU only).

The oracle (oracle/sapphire_oracle.c) is the checker of the GPU parity tests,
so it is itself checked here against the golden fixtures made by running the
reference's own kernels (tests/golden/make_golden.py), and - where the
reference library has been built in this container (oracle/_ref) - directly
against those kernels on fresh random inputs.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

from conftest import GOLDEN, normwise_rel
from oracle.oracle import Q4_0, Q8_0, TQ2_0, F32, available_reference
from sapphire_b200 import workloads

import sys
sys.path.insert(0, GOLDEN)
import make_golden  # noqa: E402  (pattern builders; no reference access at import)

# The reference AVX2 row kernel and its own scalar oracle already differ by
# 2.1e-4 absolute on bench_q4's pattern (|y| ~ 1e2); pins use normwise 1e-5.
PIN_RTOL = 1e-5


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_dispatch_row_pin(oracle, patterns):
    row, x = patterns["dispatch_row"], patterns["dispatch_x"]
    v = oracle.L.oracle_row_q4_0(row.ctypes.data, x.ctypes.data, 4)
    # test_dispatch.c:37 tolerance between kernel variants is 1e-4 absolute.
    assert abs(v - float(patterns["dispatch_unaligned"])) < 1e-5
    assert abs(v - float(patterns["dispatch_aligned"])) < 1e-5


@pytest.mark.parametrize("tag,dtype", [("bq4", Q4_0), ("bq8", Q8_0)])
def test_bench_pattern_pin(oracle, patterns, tag, dtype):
    rows, cols = patterns[f"{tag}_shape"]
    y = oracle.gemv(dtype, patterns[f"{tag}_W"], rows, cols, patterns[f"{tag}_x"])[0]
    assert normwise_rel(y, patterns[f"{tag}_y"]) < PIN_RTOL


@pytest.mark.parametrize("i", range(len(make_golden.E2E_CONFIGS)))
def test_end_to_end_pattern_pin(oracle, patterns, i):
    rows, cols = patterns[f"e2e_{i}_shape"]
    if f"e2eq4_{i}_W" in patterns:
        q4, q8 = patterns[f"e2eq4_{i}_W"], patterns[f"e2eq8_{i}_W"]
        x = (np.float32(0.001) * np.arange(1, cols + 1, dtype=np.float32)).astype(np.float32)
    else:
        q4, q8, x = make_golden.pattern_e2e(rows, cols // 32)
    for dt, W, key in ((Q4_0, q4, "q4"), (Q8_0, q8, "q8")):
        y = oracle.gemv(dt, W, rows, cols, x)[0]
        assert normwise_rel(y, patterns[f"e2e{key}_{i}_y"]) < PIN_RTOL
        # The bench prints sum(y); the float64 sum of the golden must agree.
        assert abs(y.astype(np.float64).sum() - float(patterns[f"e2e{key}_{i}_sum"])) <= \
            1e-5 * max(1.0, abs(float(patterns[f"e2e{key}_{i}_sum"])))


def test_e2e_smallest_sum_matches_reference_print(patterns):
    # bench_sapphire_end_to_end prints sum=-3.10272011 for the 64x2 Q4_0 config.
    assert abs(float(patterns["e2eq4_0_sum"]) - (-3.10272011)) < 1e-7


def test_tensor_nbytes_pins(patterns, sp):
    import ctypes
    for dt, key in ((sp.DTYPE_Q4_0, "nbytes_q4_100"), (sp.DTYPE_Q8_0, "nbytes_q8_100")):
        t = sp.lib.tensor_create(1, (ctypes.c_int * 1)(100), dt)
        assert sp.lib.tensor_nbytes(t) == int(patterns[key])
        sp.lib.tensor_release(t)


SEEDED = [("c1", workloads.C1),
          ("q8_small", workloads.GemvConfig("q8_0_4096x640", Q8_0, 4096, 640)),
          ("q4_ragged", workloads.GemvConfig("q4_0_100x80", Q4_0, 100, 80)),
          ("q8_ragged", workloads.GemvConfig("q8_0_33x70", Q8_0, 33, 70)),
          ("q4_prefill_rows", workloads.GemvConfig("q4_0_256x2560", Q4_0, 256, 2560, batch=4))]


@pytest.mark.parametrize("tag,cfg", SEEDED, ids=[t for t, _ in SEEDED])
def test_seeded_quantizer_and_gemv_pin(oracle, seeded, tag, cfg):
    w, X = workloads.make_inputs(cfg, seed=0)
    assert sha(w) == str(seeded[f"{tag}_w_sha256"]), "numpy generator stream changed"
    packed = oracle.quantize(cfg.dtype, w)
    assert sha(packed) == str(seeded[f"{tag}_packed_sha256"])
    Y = oracle.gemv(cfg.dtype, packed, cfg.rows, cfg.cols, workloads.pad_cols(X, cfg.cols))
    assert normwise_rel(Y, seeded[f"{tag}_Y"]) < PIN_RTOL


def test_ternary_fixture_pin(oracle, seeded):
    cfg = workloads.GemvConfig("tq2_0_512x1000", TQ2_0, 512, 1000)
    (trits, scales), X = workloads.make_inputs(cfg, seed=0)
    packed = oracle.pack_tq2(trits, scales)
    assert sha(packed) == str(seeded["tq2_packed_sha256"])
    Y = oracle.gemv(TQ2_0, packed, cfg.rows, cfg.cols, workloads.pad_cols(X, cfg.cols))
    assert normwise_rel(Y, seeded["tq2_Y_oracle_f64"]) < PIN_RTOL


# ---------------------------------------------------------------- formulas --
def test_q4_quantizer_formula(oracle):
    # One block by hand: largest-magnitude element -0.8 -> d = 0.1, q = trunc(x/0.1 + 8.5) capped at 15.
    v = np.zeros((1, 32), dtype=np.float32)
    v[0, :4] = [-0.8, 0.25, 0.7, 0.05]
    p = oracle.quantize(Q4_0, v)
    d = np.frombuffer(p[:4].tobytes(), dtype=np.float32)[0]
    assert d == np.float32(-0.8) / np.float32(-8.0)
    codes = [(p[4 + j // 2] >> (4 * (j & 1))) & 15 for j in range(32)]
    id_ = np.float32(1.0) / d
    exp = [min(15, int(np.float32(np.float32(x) * id_) + np.float32(8.5))) for x in v[0]]
    assert codes == exp
    assert codes[0] == 0 and codes[4] == 8


def test_q8_quantizer_formula(oracle):
    v = np.zeros((1, 32), dtype=np.float32)
    v[0, :3] = [1.27, -0.635, 0.001]
    p = oracle.quantize(Q8_0, v)
    d = np.frombuffer(p[:4].tobytes(), dtype=np.float32)[0]
    assert d == np.float32(1.27) / np.float32(127.0)
    q = p[4:].view(np.int8)
    assert q[0] == 127 and q[1] == -64 and q[2] == 0  # -63.5 rounds away from zero


def test_all_zero_block_quantizes_to_zero(oracle):
    v = np.zeros((2, 40), dtype=np.float32)
    for dt in (Q4_0, Q8_0):
        p = oracle.quantize(dt, v)
        deq = oracle.dequantize(dt, p, 2, 40)
        assert not deq.any()


def test_ternary_pack_layout(oracle):
    trits = np.array([[-1, 0, 1, 1] + [0] * 28], dtype=np.int8)
    p = oracle.pack_tq2(trits, np.array([0.5], dtype=np.float32))
    assert np.frombuffer(p[:4].tobytes(), dtype=np.float32)[0] == np.float32(0.5)
    # trit j at bits 2*(j%4) of byte j/4, code = t + 1
    assert p[4] == (0 | (1 << 2) | (2 << 4) | (2 << 6))
    assert all(b == 0x55 for b in p[5:12])


def test_dequantize_matches_definition(oracle):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((5, 70), dtype=np.float32)
    for dt in (Q4_0, Q8_0):
        p = oracle.quantize(dt, w)
        deq = oracle.dequantize(dt, p, 5, 70)
        err = np.abs(deq - w).max() / np.abs(w).max()
        assert err < (0.13 if dt == Q4_0 else 0.005)  # Q4_0 clamps +8 to +7: up to amax/8


# -------------------------------------------------- direct reference cross --
needs_ref = pytest.mark.skipif(not available_reference(), reason="oracle/_ref not built here")


@needs_ref
@pytest.mark.parametrize("dtype", [Q4_0, Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (130, 640), (64, 2560)])
def test_oracle_vs_reference_kernel(oracle, dtype, rows, cols):
    from oracle.oracle import Reference
    ref = Reference()
    ctx = ref.ctx(4)
    rng = np.random.default_rng(rows * 1000 + cols + dtype)
    w = rng.standard_normal((rows, cols), dtype=np.float32)
    x = rng.standard_normal(cols, dtype=np.float32)
    packed = oracle.quantize(dtype, w)
    y_ref = ref.gemv(ctx, dtype, packed, rows, cols, x)
    y_or = oracle.gemv(dtype, packed, rows, cols, x)[0]
    ref.L.kernel_ctx_destroy(ctx)
    assert normwise_rel(y_or, y_ref) < PIN_RTOL


@needs_ref
def test_reference_dense_gemv_matches_oracle(oracle):
    from oracle.oracle import Reference
    ref = Reference()
    ctx = ref.ctx(2)
    rng = np.random.default_rng(5)
    w = rng.standard_normal((33, 77), dtype=np.float32)
    x = rng.standard_normal(80, dtype=np.float32)
    y_ref = ref.gemv(ctx, F32, w, 33, 77, x)
    y_or = oracle.gemv(F32, w, 33, 77, x[:77])[0]
    ref.L.kernel_ctx_destroy(ctx)
    assert normwise_rel(y_or, y_ref) < PIN_RTOL
