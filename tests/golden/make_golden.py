"""Generate tests/golden/*.npz from the reference's own kernels.

Runs in the build container only (it needs oracle/_ref/libsapphire_ref.so,
compiled from the reference sources by `make -C oracle ref`).  The committed
.npz files are what the tests read; nothing at test time touches the
reference tree.

Fixtures:
  patterns.npz  - the deterministic inputs of the reference's own hot-path
                  tests and benches, restated here, with the reference's outputs:
      dispatch_*   src/test/test_dispatch.c:13-41   (4-block Q4_0 row)
      bq4_*        src/test/bench/bench_q4.c:57-70  (1024 x 8 blocks Q4_0)
      bq8_*        src/test/bench/bench_q8.c:36-42  (1024 x 8 blocks Q8_0)
      e2e{q4,q8}_{i}  src/test/bench/bench_sapphire_end_to_end.c:48-54,76-95,166-174
      nbytes_*     src/test/test_tensor.c:90-107
  seeded.npz    - seeded workloads (PCG64 seed 0) at small sizes, quantised by
                  the oracle quantiser, with the reference kernel_gemv outputs
                  and sha256 digests of the packed bytes.
Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.oracle import Oracle, Reference, Q4_0, Q8_0, TQ2_0  # noqa: E402
from sapphire_b200 import workloads  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def f32_bytes(v) -> np.ndarray:
    return np.frombuffer(np.float32(v).tobytes(), dtype=np.uint8)


def q4_block(scale, codes):
    """20-byte Q4_0 block from a scale and 32 codes (interleaved nibbles)."""
    b = np.zeros(20, dtype=np.uint8)
    b[:4] = f32_bytes(scale)
    for i in range(16):
        b[4 + i] = (codes[2 * i] & 0xF) | ((codes[2 * i + 1] & 0xF) << 4)
    return b


def q8_block(scale, codes):
    b = np.zeros(36, dtype=np.uint8)
    b[:4] = f32_bytes(scale)
    b[4:] = np.asarray(codes, dtype=np.int8).view(np.uint8)
    return b


def pattern_dispatch():
    # test_dispatch.c:13-24: scale 0.05*(1+b); byte i = (i & 15) | (((i+1) & 15) << 4)
    blocks = []
    for b in range(4):
        codes = []
        for i in range(16):
            codes += [i & 0xF, (i + 1) & 0xF]
        blocks.append(q4_block(np.float32(0.05) * np.float32(1 + b), codes))
    x = (np.float32(0.001) * np.arange(1, 129, dtype=np.float32)).astype(np.float32)
    return np.concatenate(blocks), x


def pattern_bench_q4():
    # bench_q4.c:57-70
    rows, nb = 1024, 8
    x = np.array([(i & 31) - 16 for i in range(nb * 32)], dtype=np.float32)
    W = []
    for r in range(rows):
        for b in range(nb):
            codes = []
            for i in range(16):
                codes += [(i * 2) % 16, (i * 2 + 1) % 16]
            W.append(q4_block(np.float32(0.02) * np.float32(1 + ((r + b) & 7)), codes))
    return np.concatenate(W), x, rows, nb


def pattern_bench_q8():
    # bench_q8.c:36-42
    rows, nb = 1024, 8
    x = np.array([(i & 31) - 16 for i in range(nb * 32)], dtype=np.float32)
    W = []
    for r in range(rows):
        for b in range(nb):
            W.append(q8_block(np.float32(0.02) * np.float32(1 + ((r + b) & 7)), [(i & 31) - 16 for i in range(32)]))
    return np.concatenate(W), x, rows, nb


E2E_CONFIGS = [(64, 2), (128, 4), (256, 8), (1024, 16), (8192, 32)]


def pattern_e2e(rows, nb):
    # bench_sapphire_end_to_end.c:76-95 (Q4) and :166-174 (Q8)
    x = (np.float32(0.001) * np.arange(1, nb * 32 + 1, dtype=np.float32)).astype(np.float32)
    q4, q8 = [], []
    for r in range(rows):
        for b in range(nb):
            s = np.float32(0.01) * np.float32(1 + ((r + b) & 7))
            codes = []
            for i in range(16):
                codes += [(i * 2 + 0 + r + b) & 0xF, (i * 2 + 1 + r + b) & 0xF]
            q4.append(q4_block(s, codes))
            q8.append(q8_block(s, [((i + r + b) & 0x1F) - 16 for i in range(32)]))
    return np.concatenate(q4), np.concatenate(q8), x


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ref = Reference()
    orc = Oracle()
    ctx1 = ref.ctx(1)
    ctx8 = ref.ctx(8)
    fx = {}

    row, x = pattern_dispatch()
    fx["dispatch_row"] = row
    fx["dispatch_x"] = x
    xa = np.ascontiguousarray(x)
    fx["dispatch_unaligned"] = np.float32(ref.L.quantized_gemv_q4_0_unaligned(row.ctypes.data, xa.ctypes.data, 4, 32))
    fx["dispatch_aligned"] = np.float32(ref.L.quantized_gemv_q4_0_aligned(row.ctypes.data, xa.ctypes.data, 4, 32))

    for tag, (W, xq, rows, nb) in (("bq4", pattern_bench_q4()), ("bq8", pattern_bench_q8())):
        fn = ref.L.quantized_gemv_q4_0_aligned if tag == "bq4" else ref.L.quantized_gemv_q8_0_aligned
        bsz = 20 if tag == "bq4" else 36
        y = np.array([fn(W.ctypes.data + r * nb * bsz, xq.ctypes.data, nb, 32) for r in range(rows)],
                     dtype=np.float32)
        fx[f"{tag}_W"] = W
        fx[f"{tag}_x"] = xq
        fx[f"{tag}_y"] = y
        fx[f"{tag}_shape"] = np.array([rows, nb * 32], dtype=np.int32)

    for i, (rows, nb) in enumerate(E2E_CONFIGS):
        q4, q8, xe = pattern_e2e(rows, nb)
        cols = nb * 32
        y4 = ref.gemv(ctx8, Q4_0, q4, rows, cols, xe)
        y8 = ref.gemv(ctx8, Q8_0, q8, rows, cols, xe)
        y4_1 = ref.gemv(ctx1, Q4_0, q4, rows, cols, xe)
        assert np.array_equal(y4, y4_1), "reference result depends on thread count"
        fx[f"e2eq4_{i}_y"] = y4
        fx[f"e2eq8_{i}_y"] = y8
        fx[f"e2eq4_{i}_sum"] = np.float64(y4.astype(np.float64).sum())
        fx[f"e2eq8_{i}_sum"] = np.float64(y8.astype(np.float64).sum())
        fx[f"e2e_{i}_shape"] = np.array([rows, cols], dtype=np.int32)
        if rows <= 1024:
            fx[f"e2eq4_{i}_W"] = q4
            fx[f"e2eq8_{i}_W"] = q8

    for dt, n in ((Q4_0, "q4"), (Q8_0, "q8")):
        shape = (ctypes.c_int * 1)(100)
        t = ref.L.tensor_create(1, shape, dt)
        fx[f"nbytes_{n}_100"] = np.int64(ref.L.tensor_nbytes(t))
        ref.L.tensor_release(t)
    np.savez_compressed(os.path.join(OUT, "patterns.npz"), **fx)

    # Seeded workloads at small sizes, quantised by the oracle quantiser,
    # evaluated by the reference kernel_gemv.
    sd = {}
    cases = [
        ("c1", workloads.C1),
        ("q8_small", workloads.GemvConfig("q8_0_4096x640", Q8_0, 4096, 640)),
        ("q4_ragged", workloads.GemvConfig("q4_0_100x80", Q4_0, 100, 80)),
        ("q8_ragged", workloads.GemvConfig("q8_0_33x70", Q8_0, 33, 70)),
        ("q4_prefill_rows", workloads.GemvConfig("q4_0_256x2560", Q4_0, 256, 2560, batch=4)),
    ]
    for tag, cfg in cases:
        w, X = workloads.make_inputs(cfg, seed=0)
        packed = orc.quantize(cfg.dtype, w)
        Xp = workloads.pad_cols(X, cfg.cols)
        Y = np.stack([ref.gemv(ctx8, cfg.dtype, packed, cfg.rows, cfg.cols, Xp[b]) for b in range(cfg.batch)])
        sd[f"{tag}_packed_sha256"] = np.array(sha(packed))
        sd[f"{tag}_w_sha256"] = np.array(sha(w))
        sd[f"{tag}_Y"] = Y
        sd[f"{tag}_shape"] = np.array([cfg.rows, cfg.cols, cfg.batch, cfg.dtype], dtype=np.int32)
    # Ternary: no reference kernel; the oracle's double-precision product is the
    # fixture (labelled so), with the packed digest.
    cfg = workloads.GemvConfig("tq2_0_512x1000", TQ2_0, 512, 1000)
    (trits, scales), X = workloads.make_inputs(cfg, seed=0)
    packed = orc.pack_tq2(trits, scales)
    sd["tq2_packed_sha256"] = np.array(sha(packed))
    sd["tq2_Y_oracle_f64"] = orc.gemv(TQ2_0, packed, cfg.rows, cfg.cols, workloads.pad_cols(X, cfg.cols), f64=True)
    sd["tq2_shape"] = np.array([cfg.rows, cfg.cols, 1, TQ2_0], dtype=np.int32)
    np.savez_compressed(os.path.join(OUT, "seeded.npz"), **sd)

    ref.L.kernel_ctx_destroy(ctx1)
    ref.L.kernel_ctx_destroy(ctx8)
    for f in ("patterns.npz", "seeded.npz"):
        print(f, os.path.getsize(os.path.join(OUT, f)), "bytes")


if __name__ == "__main__":
    main()
