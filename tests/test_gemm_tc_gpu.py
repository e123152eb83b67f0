"""Parity of the tensor-core batched Q4_0 product (kernel_gemm, batch >= 16).

The prefill path rounds activations to bf16 and keeps the weights exact, so
its reference result is the reference row kernel's arithmetic
((q - 8) * scale in fp32, src/kernels/q4_0_avx.c:40-41) applied to the
bf16-rounded activations: the oracle's row kernels (reference order) for the
small shapes, an f64 product of the exactly dequantised weights for the
full Gemma-3-4B FFN shape.  Tolerance: the GEMV bar, normwise 1e-4.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GEMV_RTOL, normwise_rel

pytestmark = pytest.mark.gpu

Q4_0 = 3


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def make_case(oracle, rows, cols, batch, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    packed = oracle.quantize(Q4_0, w)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    return packed, X


def padded(X, cols):
    pc = (cols + 31) // 32 * 32
    out = np.zeros((X.shape[0], pc), dtype=np.float32)
    out[:, :cols] = X
    return out


@pytest.mark.parametrize("rows,cols,batch", [
    (128, 64, 16),        # one tile, one K stage
    (256, 640, 256),      # Gemma-3-270M FFN width, one token tile
    (300, 96, 17),        # ragged rows, odd block count, ragged tokens
    (96, 2560, 40),       # fewer rows than one 128-row tile
    (384, 2560, 300),     # several token tiles with a ragged last one
    (2048, 640, 600),
    (2048, 64, 2560),     # 160 tiles: more than one wave, the last 12 run as half-width tiles
])
def test_prefill_matches_reference_rows(sp, ctx, oracle, rows, cols, batch):
    packed, X = make_case(oracle, rows, cols, batch, seed=rows + cols + batch)
    A = sp.Tensor(Q4_0, (rows, cols), packed)
    Y = sp.gemm(ctx, A, X, batch)
    ref = oracle.gemv(Q4_0, packed, rows, cols, padded(bf16_round(X), cols))
    err = normwise_rel(Y, ref)
    assert err < GEMV_RTOL, err
    # Exact weights: far below the ~1e-3 of a single bf16 weight copy.
    assert err < 2e-5, err


def test_prefill_full_shape(sp, ctx, oracle):
    """Gemma-3-4B FFN: 10240 x 2560 Q4_0 weight, 2048 tokens."""
    rows, cols, batch = 10240, 2560, 2048
    packed, X = make_case(oracle, rows, cols, batch, seed=0)
    A = sp.Tensor(Q4_0, (rows, cols), packed)
    Y = sp.gemm(ctx, A, X, batch)
    W = oracle.dequantize(Q4_0, packed, rows, cols).astype(np.float64)
    ref = bf16_round(X).astype(np.float64) @ W.T
    err = normwise_rel(Y, ref)
    assert err < GEMV_RTOL, err
    # Per token as well: every row of Y within the bar of its own scale.
    per_tok = np.max(np.abs(Y - ref), axis=1) / np.max(np.abs(ref), axis=1)
    assert per_tok.max() < GEMV_RTOL, per_tok.max()
    # Deterministic: a second call gives the same bits.
    Y2 = sp.gemm(ctx, A, X, batch)
    assert np.array_equal(Y, Y2)


def test_prefill_device_pointers(sp, ctx, oracle):
    import torch
    rows, cols, batch = 512, 640, 64
    packed, X = make_case(oracle, rows, cols, batch, seed=11)
    A = sp.Tensor(Q4_0, (rows, cols), packed)
    dev = torch.device("cuda", ctx.device)
    Xd = torch.from_numpy(X).to(dev)
    Yd = torch.full((batch, rows), float("nan"), device=dev)
    assert sp.lib.kernel_gemm_device(ctx.handle, Yd.data_ptr(), A.handle, Xd.data_ptr(), batch) == 0
    assert sp.lib.kernel_ctx_synchronize(ctx.handle) == 0
    ref = oracle.gemv(Q4_0, packed, rows, cols, padded(bf16_round(X), cols))
    assert normwise_rel(Yd.cpu().numpy(), ref) < GEMV_RTOL


def test_batch_threshold_paths_agree(sp, ctx, oracle):
    """batch 15 (per-token GEMV, fp32 activations) and 16 (tensor cores, bf16
    activations) give the same products up to the activations' bf16 rounding."""
    rows, cols = 256, 640
    packed, X = make_case(oracle, rows, cols, 16, seed=3)
    A = sp.Tensor(Q4_0, (rows, cols), packed)
    Y15 = sp.gemm(ctx, A, np.ascontiguousarray(X[:15]), 15)
    Y16 = sp.gemm(ctx, A, X, 16)
    ref32 = oracle.gemv(Q4_0, packed, rows, cols, padded(X, cols))
    assert normwise_rel(Y15, ref32[:15]) < GEMV_RTOL
    assert normwise_rel(Y16, ref32) < 1e-2          # bf16 activations


def test_fp32_products_switch(sp, ctx, oracle):
    """kernel_ctx_set_fp32_products(ctx, 1): a batch-32 Q4_0 kernel_gemm keeps
    fp32 activations - each row equals kernel_gemv of that row bit for bit and
    matches the oracle on the unrounded activations; switched off again, the
    same call runs the bf16 tensor-core product."""
    from conftest import GEMV_RTOL, normwise_rel
    from sapphire_b200 import workloads
    rows, cols, batch = 1024, 640, 32
    rng = np.random.default_rng(17)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    packed = oracle.quantize(sp.DTYPE_Q4_0, w)
    A = sp.Tensor(sp.DTYPE_Q4_0, (rows, cols), packed)
    X = rng.standard_normal((batch, cols), dtype=np.float32)
    ref = oracle.gemv(sp.DTYPE_Q4_0, packed, rows, cols, workloads.pad_cols(X, cols), f64=True)
    assert sp.lib.kernel_ctx_set_fp32_products(ctx.handle, 1) == 0
    try:
        Y = sp.gemm(ctx, A, X, batch)
        for b in range(batch):
            assert np.array_equal(Y[b], sp.gemv(ctx, A, X[b])), b
            assert normwise_rel(Y[b], ref[b]) < GEMV_RTOL
    finally:
        assert sp.lib.kernel_ctx_set_fp32_products(ctx.handle, 0) == 0
    Yb = sp.gemm(ctx, A, X, batch)
    assert not np.array_equal(Yb, Y)        # bf16 activations on the tensor cores
    assert normwise_rel(Yb, ref) < 1e-2
