"""kernel_gemv_device_noalloc: the batch-1 GEMV for callers that may not
allocate device memory while they multiply (fixed-budget serving loops,
paths where an allocation's implicit synchronisation would stall other work).

Its output must match kernel_gemv_device (the allocating entry point) within
the GEMV tolerance, on two calls in a row (the second call reuses the shared
scratch array left by the first).  This file is collected last so that a run
stopping at the first failure has already run every other test; it also
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


@pytest.mark.parametrize("dtype_name,rows,cols", [("Q8_0", 262144, 640), ("Q4_0", 4096, 2560),
                                                  ("TQ2_0", 2048, 4096), ("Q8_0", 33, 70)])
def test_noalloc_matches_allocating_entry_point(nctx, dtype_name, rows, cols):
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
        nctx.synchronize()
        assert torch.isfinite(y).all()
        assert normwise_rel(y.cpu().numpy(), y_ref.cpu().numpy()) < GEMV_RTOL
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
