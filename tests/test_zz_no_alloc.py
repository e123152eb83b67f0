"""kernel_gemv_device_noalloc: the batch-1 GEMV for callers that may not
allocate device memory while they multiply - a serving loop that owns a fixed
memory budget or pool, or a path where an allocation's implicit device
synchronisation would stall other streams.  They upload their weights at load
time (kernel_tensor_upload allocates) and then multiply with this entry point,
whose scratch is a fixed array inside the library.

Checked here, through the C-ABI: the output matches the allocating entry
point (kernel_gemv_device) and the oracle within the GEMV bar on two calls in
a row (the second reuses the scratch the first left behind); repeated calls
leave the device's free memory unchanged; what it cannot serve is refused;
and a kernel error (an expired bounded wait, made to happen with a test hook)
is reported by the next kernel_ctx_synchronize instead of being lost, after
which the entry point is correct again.  This file is collected last so that a
run stopping at the first failure has already run every other test; it also
passes alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GEMV_RTOL, normwise_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nctx():
    import sapphire_b200 as sp
    c = sp.Context(num_threads=1)
    yield c
    c.close()


def packed_weight(sp, dtype, rows, cols, seed):
    rng = np.random.default_rng(seed)
    if dtype == sp.DTYPE_TQ2_0:
        trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
        return sp.pack_tq2(None, trits, rng.uniform(0.01, 0.1, size=rows).astype(np.float32))
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    return sp.quantize(None, dtype, w)


def oracle_y(dtype, packed, rows, cols, x):
    from oracle.oracle import Oracle
    xp = np.zeros((1, (cols + 31) // 32 * 32), dtype=np.float32)
    xp[0, :cols] = x
    return Oracle().gemv(dtype, packed, rows, cols, xp, f64=True)[0]


@pytest.mark.parametrize("dtype_name,rows,cols", [("Q8_0", 262144, 640), ("Q4_0", 4096, 2560),
                                                  ("TQ2_0", 2048, 4096), ("Q8_0", 33, 70)])
def test_noalloc_matches_allocating_entry_point_and_oracle(nctx, dtype_name, rows, cols):
    import torch
    import sapphire_b200 as sp
    dtype = getattr(sp, f"DTYPE_{dtype_name}")
    packed = packed_weight(sp, dtype, rows, cols, seed=rows + cols)
    A = sp.Tensor(dtype, (rows, cols), packed)
    L, h = sp.lib, nctx.handle
    assert L.kernel_tensor_upload(h, A.handle) == 0           # allocation happens here, at load
    y_ref = torch.empty(rows, device="cuda")
    y = torch.empty(rows, device="cuda")
    for call in range(2):
        x = torch.randn(cols, device="cuda", generator=torch.Generator("cuda").manual_seed(call))
        assert L.kernel_gemv_device(h, y_ref.data_ptr(), A.handle, x.data_ptr()) == 0
        y.fill_(float("nan"))
        assert L.kernel_gemv_device_noalloc(h, y.data_ptr(), A.handle, x.data_ptr()) == 0
        assert L.kernel_ctx_synchronize(h) == 0
        assert torch.isfinite(y).all()
        yn = y.cpu().numpy()
        assert normwise_rel(yn, y_ref.cpu().numpy()) < GEMV_RTOL
        assert normwise_rel(yn, oracle_y(dtype, packed, rows, cols, x.cpu().numpy())) < GEMV_RTOL
    assert L.kernel_tensor_evict(h, A.handle) == 0


def test_noalloc_leaves_device_memory_unchanged():
    # A fresh context that never runs the allocating entry point: after the
    # weight upload and one warm-up call, repeated calls change nothing in the
    # device's free memory.
    import torch
    import sapphire_b200 as sp
    with sp.Context(num_threads=1) as c:
        rows, cols = 65536, 640
        packed = packed_weight(sp, sp.DTYPE_Q4_0, rows, cols, seed=3)
        A = sp.Tensor(sp.DTYPE_Q4_0, (rows, cols), packed)
        assert sp.lib.kernel_tensor_upload(c.handle, A.handle) == 0
        x = torch.randn(cols, device="cuda")
        y = torch.empty(rows, device="cuda")
        assert sp.lib.kernel_gemv_device_noalloc(c.handle, y.data_ptr(), A.handle, x.data_ptr()) == 0
        assert sp.lib.kernel_ctx_synchronize(c.handle) == 0
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        for _ in range(20):
            assert sp.lib.kernel_gemv_device_noalloc(c.handle, y.data_ptr(), A.handle, x.data_ptr()) == 0
        assert sp.lib.kernel_ctx_synchronize(c.handle) == 0
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0
        assert normwise_rel(y.cpu().numpy(), oracle_y(sp.DTYPE_Q4_0, packed, rows, cols, x.cpu().numpy())) \
            < GEMV_RTOL
        A.release()


def test_noalloc_reports_kernel_errors(nctx):
    import torch
    import sapphire_b200 as sp
    L, h = sp.lib, nctx.handle
    rows, cols = 32768, 640
    packed = packed_weight(sp, sp.DTYPE_Q8_0, rows, cols, seed=5)
    A = sp.Tensor(sp.DTYPE_Q8_0, (rows, cols), packed)
    assert L.kernel_tensor_upload(h, A.handle) == 0
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    L.sapphire_test_stream_unarmed(1)
    try:
        assert L.kernel_gemv_device_noalloc(h, y.data_ptr(), A.handle, x.data_ptr()) == 0   # enqueued
        rc = L.kernel_ctx_synchronize(h)
    finally:
        L.sapphire_test_stream_unarmed(0)
    assert rc == -1
    assert "bounded wait expired" in nctx.last_error
    for _ in range(2):
        assert L.kernel_gemv_device_noalloc(h, y.data_ptr(), A.handle, x.data_ptr()) == 0
        assert L.kernel_ctx_synchronize(h) == 0
        assert normwise_rel(y.cpu().numpy(), oracle_y(sp.DTYPE_Q8_0, packed, rows, cols, x.cpu().numpy())) \
            < GEMV_RTOL
    assert L.kernel_tensor_evict(h, A.handle) == 0


def test_noalloc_rejects_what_it_cannot_serve(nctx):
    import torch
    import sapphire_b200 as sp
    L, h = sp.lib, nctx.handle
    x = torch.randn(32, device="cuda")
    y = torch.empty(1 << 20, device="cuda")
    # Not resident: the entry point must not upload (that would allocate).
    small = sp.Tensor(sp.DTYPE_Q8_0, (64, 32), packed_weight(sp, sp.DTYPE_Q8_0, 64, 32, seed=1))
    assert L.kernel_gemv_device_noalloc(h, y.data_ptr(), small.handle, x.data_ptr()) == -1
    assert "not resident" in nctx.last_error
    # 2^20 rows x 32 columns needs more than the fixed 4 MiB of scratch.
    big = sp.Tensor(sp.DTYPE_Q8_0, (1 << 20, 32), packed_weight(sp, sp.DTYPE_Q8_0, 1 << 20, 32, seed=2))
    assert L.kernel_tensor_upload(h, big.handle) == 0
    assert L.kernel_gemv_device_noalloc(h, y.data_ptr(), big.handle, x.data_ptr()) == -1
    assert "maximum" in nctx.last_error
    # Host pointers are refused.
    xh = np.ones(32, dtype=np.float32)
    assert L.kernel_gemv_device_noalloc(h, y.data_ptr(), big.handle, xh.ctypes.data) == -1
    assert L.kernel_tensor_evict(h, big.handle) == 0
