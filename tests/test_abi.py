"""C-ABI checks that need no GPU: the library loads, exports every entry point
the headers declare, and the host-side tensor API and argument checks behave
like the reference (src/tensor/tensor.c, src/kernels/dispatch.c)."""
from __future__ import annotations

import ctypes as C
import glob
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))

# Every function of the reference's hot-path headers (include/kernels.h:56-166,
# include/tensor.h:60-208) that a drop-in must export.
REFERENCE_API = """
kernel_ctx_create kernel_ctx_init kernel_ctx_destroy kernel_parallel_for
quantized_gemv_q4_0_aligned quantized_gemv_q4_0_unaligned quantized_gemv_q8_0_aligned
quantized_gemv_q8_0_unaligned quantized_gemv_bf16_avx2 quantized_gemv_bf16_scalar
quantized_gemv_f32_avx2 quantized_gemv_f32_scalar kernel_gemm_f32_avx2 kernel_gemm_bf16_avx2
kernel_gemv kernel_gemm kernel_gemv_tensor kernel_gemv_add kernel_gemv_batch kernel_get_simd_lane_count
tensor_create tensor_transpose tensor_clone tensor_numel dtype_element_size dtype_name tensor_get_f32
tensor_set_f32 tensor_ref_inc tensor_release tensor_print_info tensor_ndim tensor_shape tensor_data
tensor_data_f32 tensor_data_mutable tensor_dtype tensor_nbytes tensor_ref_count tensor_create_view
""".split()


def declared_api() -> set[str]:
    names = set()
    for h in HEADERS:
        for m in re.finditer(r"^SAPPHIRE_API\s+[^;(]*?\b(\w+)\s*\(", open(h).read(), re.M):
            names.add(m.group(1))
    return names


def exported(path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_library_loads_and_exports_every_declared_symbol(sp):
    from sapphire_b200._lib import LIB_PATH, exported_names
    decl = declared_api()
    assert len(decl) >= 60
    exp = exported(LIB_PATH)
    missing = sorted(decl - exp)
    assert not missing, f"declared but not exported: {missing}"
    # The Python mirror binds exactly the declared set.
    assert set(exported_names()) == decl
    for name in decl:
        assert getattr(sp.lib, name) is not None


def test_reference_api_is_complete():
    missing = sorted(set(REFERENCE_API) - declared_api())
    assert not missing, missing


def test_host_helpers_not_claimed_as_exports():
    # rmsnorm & co. are declared for source compatibility only.
    decl = declared_api()
    for n in ("rmsnorm", "rmsnorm_delta", "gelu", "softmax", "vec_dot"):
        assert n not in decl


def test_no_oracle_in_product():
    from sapphire_b200._lib import LIB_PATH
    out = subprocess.run(["nm", "-D", LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "oracle_" not in out
    deps = subprocess.run(["ldd", LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in deps and "sapphire_ref" not in deps


# ------------------------------------------------------------- tensor API --
def shape_arr(*s):
    return (C.c_int * len(s))(*s)


def test_tensor_create_byte_counts(sp):
    L = sp.lib
    cases = [(sp.DTYPE_F32, (3, 4), 48), (sp.DTYPE_BF16, (5,), 10), (sp.DTYPE_Q4_0, (100,), 50),
             (sp.DTYPE_Q4_0, (7,), 4), (sp.DTYPE_Q8_0, (100,), 100), (sp.DTYPE_TQ2_0, (64,), 64)]
    for dt, shape, nbytes in cases:
        t = L.tensor_create(len(shape), shape_arr(*shape), dt)
        assert t
        assert L.tensor_nbytes(t) == nbytes
        assert L.tensor_ndim(t) == len(shape)
        assert L.tensor_numel(t) == int(np.prod(shape))
        assert L.tensor_ref_count(t) == 1
        L.tensor_release(t)


def test_tensor_create_rejects_bad_ndim(sp):
    assert not sp.lib.tensor_create(0, shape_arr(1), sp.DTYPE_F32)
    assert not sp.lib.tensor_create(9, shape_arr(*([1] * 9)), sp.DTYPE_F32)
    assert not sp.lib.tensor_create(2, None, sp.DTYPE_F32)


def test_tensor_get_set_transpose_clone(sp):
    L = sp.lib
    t = L.tensor_create(2, shape_arr(2, 3), sp.DTYPE_F32)
    for i in range(6):
        assert L.tensor_set_f32(t, i, float(i)) == 0
    assert L.tensor_set_f32(t, 6, 1.0) == -1
    assert L.tensor_get_f32(t, 4) == 4.0
    out = C.c_void_p()
    assert L.tensor_transpose(t, C.byref(out)) == 0
    tt = out.value
    assert list(L.tensor_shape(tt)[:2]) == [3, 2]
    assert L.tensor_get_f32(tt, 1) == 3.0   # [0][1] of transpose = [1][0] of source
    c = L.tensor_clone(t)
    assert L.tensor_get_f32(c, 5) == 5.0 and L.tensor_data(c) != L.tensor_data(t)
    L.tensor_ref_inc(t)
    assert L.tensor_ref_count(t) == 2
    L.tensor_release(t)
    assert L.tensor_ref_count(t) == 1
    for h in (t, tt, c):
        L.tensor_release(h)


def test_tensor_quantized_element_access_is_stubbed(sp):
    L = sp.lib
    t = L.tensor_create(1, shape_arr(64), sp.DTYPE_Q8_0)
    assert L.tensor_get_f32(t, 0) == 0.0          # reference tensor.c:238-244
    assert L.tensor_set_f32(t, 0, 1.0) == -1
    assert not L.tensor_data_f32(t)
    L.tensor_release(t)


def test_views_are_non_owning(sp):
    buf = np.arange(8, dtype=np.float32)
    t = sp.Tensor(sp.DTYPE_F32, (2, 4), buf)
    assert sp.lib.tensor_data(t.handle) == buf.ctypes.data
    assert sp.lib.tensor_nbytes(t.handle) == 32
    t.release()
    assert buf[3] == 3.0


def test_null_safety(sp):
    L = sp.lib
    assert L.tensor_ndim(None) == 0 and L.tensor_numel(None) == 0 and L.tensor_nbytes(None) == 0
    assert not L.tensor_shape(None) and not L.tensor_data(None)
    assert L.tensor_dtype(None) == sp.DTYPE_F32
    L.tensor_release(None)
    L.kernel_ctx_destroy(None)
    assert L.dtype_name(sp.DTYPE_TQ2_0) == b"TQ2_0" and L.dtype_name(99) == b"UNKNOWN"
    # Additive entry points refuse a NULL handle instead of touching it.
    assert L.kernel_ctx_set_fp32_products(None, 1) == -1
    assert L.sapphire_decoder_launches_per_token(None) == -1
    assert L.sapphire_decoder_launches_per_prompt_token(None) == -1
    assert L.sapphire_decoder_generate(None, None, 0, 0, None, None) == -1
    L.sapphire_decoder_destroy(None)
    assert L.sapphire_safetensors_count(None) == -1 and not L.sapphire_safetensors_name(None, 0)
    assert not L.sapphire_safetensors_tensor(None, b"x") and not L.sapphire_safetensors_open(None)
    L.sapphire_safetensors_close(None)
    assert not L.sapphire_decoder_create_from_safetensors(None, None, None)


def test_simd_lane_count(sp):
    for dt in (sp.DTYPE_F32, sp.DTYPE_BF16, sp.DTYPE_F16, sp.DTYPE_Q4_0, sp.DTYPE_Q8_0, sp.DTYPE_TQ2_0):
        assert sp.lib.kernel_get_simd_lane_count(dt) == 8
    assert sp.lib.kernel_get_simd_lane_count(42) == 1


def test_row_bytes(sp):
    assert sp.row_bytes(sp.DTYPE_Q4_0, 640) == 400
    assert sp.row_bytes(sp.DTYPE_Q8_0, 640) == 720
    assert sp.row_bytes(sp.DTYPE_TQ2_0, 16384) == 4100
    assert sp.row_bytes(sp.DTYPE_Q4_0, 33) == 40


# ------------------------------------------------------- argument checks ---
def test_gemv_argument_errors_before_any_gpu_work(sp):
    L = sp.lib
    w = np.zeros(4 * 8, dtype=np.float32)
    A = sp.Tensor(sp.DTYPE_F32, (4, 8), w)
    A1 = sp.Tensor(sp.DTYPE_F32, (32,), w)
    Aq = sp.Tensor(sp.DTYPE_Q4_0, (4, 32), np.zeros(80, dtype=np.uint8))
    x = np.zeros(32, dtype=np.float32)
    y = np.zeros(4, dtype=np.float32)
    assert L.kernel_gemv(None, None, A.handle, x.ctypes.data) == -1
    assert L.kernel_gemv(None, y.ctypes.data, None, x.ctypes.data) == -1
    assert L.kernel_gemv(None, y.ctypes.data, A.handle, None) == -1
    assert L.kernel_gemv(None, y.ctypes.data, A1.handle, x.ctypes.data) == -1
    # quantized weights need a context (reference dispatch.c:140-141)
    assert L.kernel_gemv(None, y.ctypes.data, Aq.handle, x.ctypes.data) == -1
    assert L.kernel_gemm(None, y.ctypes.data, A.handle, x.ctypes.data, 1, 4) == -1
    assert L.kernel_gemm(None, y.ctypes.data, A.handle, x.ctypes.data, 0, 4) == -1
    assert L.kernel_gemv_batch(None, y.ctypes.data, A.handle, x.ctypes.data, 0) == -1
    assert L.kernel_gemv_add(None, None, A.handle, x.ctypes.data, 1.0) == -1
    assert L.kernel_gemv_add(None, y.ctypes.data, A1.handle, x.ctypes.data, 1.0) == -1


def test_gemv_tensor_shape_checks(sp):
    L = sp.lib
    A = L.tensor_create(2, shape_arr(3, 4), sp.DTYPE_F32)
    x_bad = L.tensor_create(1, shape_arr(5), sp.DTYPE_F32)
    y = L.tensor_create(1, shape_arr(3), sp.DTYPE_F32)
    y_bad = L.tensor_create(1, shape_arr(2), sp.DTYPE_F32)
    x = L.tensor_create(1, shape_arr(4), sp.DTYPE_F32)
    x2d = L.tensor_create(2, shape_arr(1, 4), sp.DTYPE_F32)
    assert L.kernel_gemv_tensor(None, y, A, x_bad) == -1
    assert L.kernel_gemv_tensor(None, y_bad, A, x) == -1
    assert L.kernel_gemv_tensor(None, y, A, x2d) == -1
    assert L.kernel_gemv_tensor(None, None, A, x) == -1
    for h in (A, x_bad, y, y_bad, x, x2d):
        L.tensor_release(h)


def test_parallel_for_runs_every_index(sp):
    L = sp.lib
    ctx = L.kernel_ctx_create(3, 16)
    L.kernel_ctx_init(ctx)   # fails on a machine without a GPU; workers then run inline
    seen = np.zeros(100, dtype=np.int32)

    @sp.PARALLEL_FOR_FN
    def body(arg, i):
        seen[i] += 1

    assert L.kernel_parallel_for(ctx, body, None, 100) == 0
    assert (seen == 1).all()
    assert L.kernel_parallel_for(ctx, body, None, 0) == -1
    assert L.kernel_parallel_for(None, body, None, 5) == -1
    L.kernel_ctx_destroy(ctx)


def test_init_without_gpu_fails_loudly(sp):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = sp.lib.kernel_ctx_create(1, 16)
    assert sp.lib.kernel_ctx_init(ctx) == -1
    assert b"no CUDA device" in sp.lib.kernel_ctx_last_error(ctx)
    sp.lib.kernel_ctx_destroy(ctx)
