"""Bounded device waits made to run out on purpose, without any GPU fault.

Every device wait of the library is bounded; a wait that runs out records a
bit in the context's error word and the kernel returns, so the host call fails
with -1 and the context stays usable.  These tests make a wait run out with a
barrier or a flag that nothing sets (test hooks in include/sapphire_cuda.h)
and check the status, the message and that the next products are correct:

* the streaming GEMV: one consumer warp's first shared-memory slot is never
  filled (its copy is not issued) and its wait has a short limit.  The warps
  that shared tiles with it leave their arrival counts behind; the library
  clears the counters when it reports the error, which the following products
  prove by matching the oracle bit for bit with an earlier result;
* the peer-memory gather of sharded products: the pull waits on a local
  buffer that no rank writes, with a 1 ms limit.  Once one word has expired a
  block stops waiting for the others, so even 4M rows end within the limit's
  order of magnitude, not one limit per word.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from conftest import GEMV_RTOL, normwise_rel
from oracle.oracle import Q8_0, TQ2_0
from sapphire_b200 import workloads

pytestmark = pytest.mark.gpu


def _weight(oracle, dtype, rows, cols, seed):
    rng = np.random.default_rng(seed)
    if dtype == TQ2_0:
        trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
        return oracle.pack_tq2(trits, rng.uniform(0.01, 0.1, size=rows).astype(np.float32))
    return oracle.quantize(dtype, (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))


@pytest.mark.parametrize("dtype,rows,cols", [(Q8_0, 32768, 640), (TQ2_0, 4096, 4096)])
def test_stream_wait_expiry_reports_and_recovers(sp, ctx, oracle, dtype, rows, cols):
    import torch
    packed = _weight(oracle, dtype, rows, cols, seed=rows)
    x = np.random.default_rng(cols).standard_normal(cols, dtype=np.float32)
    A = sp.Tensor(dtype, (rows, cols), packed)
    ref = oracle.gemv(dtype, packed, rows, cols, workloads.pad_cols(x[None], cols), f64=True)[0]
    y0 = sp.gemv(ctx, A, x)
    assert normwise_rel(y0, ref) < GEMV_RTOL
    L = sp.lib
    # Synchronous entry point: the call itself fails.
    L.sapphire_test_stream_unarmed(1)
    try:
        yb = np.zeros(rows, dtype=np.float32)
        rc = L.kernel_gemv(ctx.handle, yb.ctypes.data, A.handle, x.ctypes.data)
    finally:
        L.sapphire_test_stream_unarmed(0)
    assert rc == -1
    assert "bounded wait expired" in ctx.last_error
    for _ in range(2):
        assert np.array_equal(sp.gemv(ctx, A, x), y0)
    # Asynchronous entry point: the error surfaces at kernel_ctx_synchronize.
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros(rows, device="cuda")
    L.sapphire_test_stream_unarmed(1)
    try:
        assert L.kernel_gemv_device(ctx.handle, yd.data_ptr(), A.handle, xd.data_ptr()) == 0
        rc = L.kernel_ctx_synchronize(ctx.handle)
    finally:
        L.sapphire_test_stream_unarmed(0)
    assert rc == -1
    assert "bounded wait expired" in ctx.last_error
    assert L.kernel_ctx_synchronize(ctx.handle) == 0                  # reported once, then cleared
    assert L.kernel_gemv_device(ctx.handle, yd.data_ptr(), A.handle, xd.data_ptr()) == 0
    assert L.kernel_ctx_synchronize(ctx.handle) == 0
    assert np.array_equal(yd.cpu().numpy(), y0)
    A.release()


@pytest.mark.parametrize("rows", [1000, 1 << 22])
def test_peer_gather_wait_expiry(sp, ctx, rows):
    import torch
    y = torch.zeros(rows, device="cuda")
    t0 = time.perf_counter()
    rc = sp.lib.sapphire_test_pull_expiry(ctx.handle, y.data_ptr(), rows, 1_000_000)   # 1 ms limit
    elapsed = time.perf_counter() - t0
    assert rc == -1
    assert "peer-memory gather" in ctx.last_error
    assert torch.isnan(y).all()
    assert elapsed < 2.0, elapsed
    # The context is still usable.
    assert sp.lib.kernel_ctx_synchronize(ctx.handle) == 0
    A = sp.Tensor(Q8_0, (64, 64), np.zeros(64 * 2 * 36, dtype=np.uint8))
    assert np.array_equal(sp.gemv(ctx, A, np.ones(64, dtype=np.float32)), np.zeros(64, dtype=np.float32))
