"""ctypes binding of libsapphire_cuda.so (the C-ABI in include/*.h).

The library is loaded from this package folder.  There is no fallback: if the
shared object is missing, importing the binding raises, naming the build step.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsapphire_cuda.so")

# tensor_dtype_t (include/tensor.h)
DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_Q4_0, DTYPE_Q8_0, DTYPE_TQ2_0 = range(6)
DTYPE_NAMES = {DTYPE_F32: "F32", DTYPE_BF16: "BF16", DTYPE_F16: "F16", DTYPE_Q4_0: "Q4_0",
               DTYPE_Q8_0: "Q8_0", DTYPE_TQ2_0: "TQ2_0"}
UNIQUE_ID_BYTES = 128

vp = C.c_void_p
i32 = C.c_int
f32 = C.c_float
sz = C.c_size_t

PARALLEL_FOR_FN = C.CFUNCTYPE(None, vp, i32)


class GemmArgs(C.Structure):
    """gemm_args_t (include/kernels.h)."""
    _fields_ = [("w_row", vp), ("X", vp), ("Y", vp), ("batch_size", i32), ("d_model", i32),
                ("out_stride", i32), ("blocks", i32), ("block_size", i32)]


# name: (restype, argtypes)
_SIGNATURES = {
    # include/tensor.h
    "tensor_create": (vp, [i32, C.POINTER(i32), i32]),
    "tensor_transpose": (i32, [vp, C.POINTER(vp)]),
    "tensor_clone": (vp, [vp]),
    "tensor_numel": (sz, [vp]),
    "dtype_element_size": (sz, [i32]),
    "dtype_name": (C.c_char_p, [i32]),
    "tensor_get_f32": (f32, [vp, sz]),
    "tensor_set_f32": (i32, [vp, sz, f32]),
    "tensor_ref_inc": (None, [vp]),
    "tensor_release": (None, [vp]),
    "tensor_print_info": (None, [vp]),
    "tensor_ndim": (i32, [vp]),
    "tensor_shape": (C.POINTER(i32), [vp]),
    "tensor_data": (vp, [vp]),
    "tensor_data_f32": (vp, [vp]),
    "tensor_data_mutable": (vp, [vp]),
    "tensor_dtype": (i32, [vp]),
    "tensor_nbytes": (sz, [vp]),
    "tensor_ref_count": (i32, [vp]),
    "tensor_create_view": (vp, [i32, i32, C.POINTER(i32), vp]),
    # include/kernels.h
    "kernel_ctx_create": (vp, [i32, i32]),
    "kernel_ctx_init": (i32, [vp]),
    "kernel_ctx_destroy": (None, [vp]),
    "kernel_parallel_for": (i32, [vp, PARALLEL_FOR_FN, vp, i32]),
    "quantized_gemv_q4_0_aligned": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_q4_0_unaligned": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_q8_0_aligned": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_q8_0_unaligned": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_bf16_avx2": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_bf16_scalar": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_f32_avx2": (f32, [vp, vp, i32, i32]),
    "quantized_gemv_f32_scalar": (f32, [vp, vp, i32, i32]),
    "kernel_gemm_f32_avx2": (None, [C.POINTER(GemmArgs)]),
    "kernel_gemm_bf16_avx2": (None, [C.POINTER(GemmArgs)]),
    "kernel_gemv": (i32, [vp, vp, vp, vp]),
    "kernel_gemm": (i32, [vp, vp, vp, vp, i32, i32]),
    "kernel_gemv_tensor": (i32, [vp, vp, vp, vp]),
    "kernel_gemv_add": (i32, [vp, vp, vp, vp, f32]),
    "kernel_gemv_batch": (i32, [vp, vp, vp, vp, i32]),
    "kernel_get_simd_lane_count": (i32, [i32]),
    # include/sapphire_cuda.h
    "quantized_gemv_tq2_0": (f32, [vp, vp, i32, i32]),
    "sapphire_row_bytes": (sz, [i32, i32]),
    "kernel_tensor_upload": (i32, [vp, vp]),
    "kernel_tensor_evict": (i32, [vp, vp]),
    "kernel_ctx_resident_bytes": (sz, [vp]),
    "kernel_gemv_device": (i32, [vp, vp, vp, vp]),
    "kernel_gemv_device_noalloc": (i32, [vp, vp, vp, vp]),
    "kernel_gemm_device": (i32, [vp, vp, vp, vp, i32]),
    "kernel_gemm_device_bf16": (i32, [vp, vp, vp, vp, i32, i32]),
    "sapphire_shard_rows": (i32, [i32, i32, i32, vp, vp]),
    "kernel_ctx_synchronize": (i32, [vp]),
    "kernel_ctx_set_device": (i32, [vp, i32]),
    "kernel_ctx_set_fp32_products": (i32, [vp, i32]),
    "kernel_ctx_get_stream": (vp, [vp]),
    "kernel_ctx_set_stream": (i32, [vp, vp]),
    "kernel_ctx_get_device": (i32, [vp]),
    "kernel_ctx_last_error": (C.c_char_p, [vp]),
    "kernel_host_alloc": (vp, [sz]),
    "kernel_host_free": (None, [vp]),
    "kernel_quantize_q4_0": (i32, [vp, vp, vp, i32, i32]),
    "kernel_quantize_q8_0": (i32, [vp, vp, vp, i32, i32]),
    "kernel_pack_tq2_0": (i32, [vp, vp, vp, vp, i32, i32]),
    "kernel_dequantize": (i32, [vp, vp, vp]),
    "kernel_shard_unique_id": (i32, [vp]),
    "kernel_ctx_init_sharded": (i32, [vp, i32, i32, vp]),
    "kernel_ctx_shard_info": (i32, [vp, C.POINTER(i32), C.POINTER(i32)]),
    "sapphire_test_stream_unarmed": (i32, [i32]),
    "sapphire_test_pull_expiry": (i32, [vp, vp, C.c_longlong, C.c_ulonglong]),
    # include/sapphire_safetensors.h
    "sapphire_safetensors_open": (vp, [C.c_char_p]),
    "sapphire_safetensors_count": (i32, [vp]),
    "sapphire_safetensors_name": (C.c_char_p, [vp, i32]),
    "sapphire_safetensors_tensor": (vp, [vp, C.c_char_p]),
    "sapphire_safetensors_close": (None, [vp]),
    "sapphire_decoder_create_from_safetensors": (vp, [vp, vp, vp]),
    "sapphire_test_decode_stall": (i32, [i32]),
    # include/sapphire_decode.h
    "sapphire_decoder_create": (vp, [vp, vp, vp]),
    "sapphire_decoder_generate": (i32, [vp, vp, i32, i32, vp, vp]),
    "sapphire_decoder_last_logits": (i32, [vp, vp]),
    "sapphire_decoder_last_times": (i32, [vp, C.POINTER(f32), C.POINTER(f32)]),
    "sapphire_decoder_launches_per_token": (i32, [vp]),
    "sapphire_decoder_launches_per_prompt_token": (i32, [vp]),
    "sapphire_decoder_destroy": (None, [vp]),
}


class Gemma3Config(C.Structure):
    """sapphire_gemma3_config_t (include/sapphire_decode.h)."""
    _fields_ = [("layers", i32), ("hidden", i32), ("ffn", i32), ("heads", i32), ("kv_heads", i32),
                ("head_dim", i32), ("vocab", i32), ("context", i32), ("sliding_window", i32),
                ("rope_theta", f32), ("rope_local_theta", f32), ("query_pre_attn_scalar", f32),
                ("rms_eps", f32), ("global_mask", C.c_ulonglong)]


class Gemma3Weights(C.Structure):
    """sapphire_gemma3_weights_t (include/sapphire_decode.h)."""
    _fields_ = [("embed_bf16", vp), ("lm_head", vp), ("final_norm", vp), ("proj", vp), ("norms", vp)]


def load(path: str = LIB_PATH) -> C.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `make -C sapphire_b200/csrc` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def exported_names() -> list[str]:
    return sorted(_SIGNATURES)
