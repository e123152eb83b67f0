"""ctypes access to the test-side checkers.  TEST INFRASTRUCTURE ONLY.

`Oracle` wraps oracle/liboracle.so (the C restatement, sapphire_oracle.c).
`Reference` wraps oracle/_ref/libsapphire_ref.so: the reference's own C
sources compiled unmodified by oracle/Makefile.  Only tests/, the smoke check
and bench.py's CPU-baseline leg use this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsapphire_ref.so")

F32, BF16, F16, Q4_0, Q8_0, TQ2_0 = range(6)

vp, i32, f32 = C.c_void_p, C.c_int, C.c_float


def _a(x) -> int:
    return x.ctypes.data if isinstance(x, np.ndarray) else int(x or 0)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = C.CDLL(path)
        L.oracle_row_bytes.restype = C.c_size_t
        L.oracle_row_bytes.argtypes = [i32, i32]
        for n in ("oracle_row_q4_0", "oracle_row_q8_0", "oracle_row_tq2_0"):
            getattr(L, n).restype = f32
            getattr(L, n).argtypes = [vp, vp, i32]
        L.oracle_gemv.argtypes = [i32, vp, i32, i32, vp, i32, vp, i32]
        L.oracle_gemv_f64.argtypes = [i32, vp, i32, i32, vp, i32, vp, i32]
        L.oracle_quantize.argtypes = [i32, vp, i32, i32, vp]
        L.oracle_pack_tq2_0.argtypes = [vp, vp, i32, i32, vp]
        L.oracle_dequantize.argtypes = [i32, vp, i32, i32, vp]
        self.L = L

    def row_bytes(self, dtype: int, cols: int) -> int:
        return int(self.L.oracle_row_bytes(dtype, cols))

    def quantize(self, dtype: int, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(rows * self.row_bytes(dtype, cols), dtype=np.uint8)
        assert self.L.oracle_quantize(dtype, _a(w), rows, cols, _a(out)) == 0
        return out

    def pack_tq2(self, trits: np.ndarray, scales: np.ndarray) -> np.ndarray:
        trits = np.ascontiguousarray(trits, dtype=np.int8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        rows, cols = trits.shape
        out = np.zeros(rows * self.row_bytes(TQ2_0, cols), dtype=np.uint8)
        assert self.L.oracle_pack_tq2_0(_a(trits), _a(scales), rows, cols, _a(out)) == 0
        return out

    def dequantize(self, dtype: int, packed: np.ndarray, rows: int, cols: int) -> np.ndarray:
        out = np.zeros((rows, cols), dtype=np.float32)
        assert self.L.oracle_dequantize(dtype, _a(packed), rows, cols, _a(out)) == 0
        return out

    def gemv(self, dtype: int, packed, rows: int, cols: int, X: np.ndarray, f64: bool = False,
             nthreads: int = 0) -> np.ndarray:
        """Y[b, r]; X is [batch, padded cols] (zero-padded to a multiple of 32)."""
        X = np.ascontiguousarray(np.atleast_2d(X), dtype=np.float32)
        batch = X.shape[0]
        Y = np.zeros((batch, rows), dtype=np.float64 if f64 else np.float32)
        fn = self.L.oracle_gemv_f64 if f64 else self.L.oracle_gemv
        assert fn(dtype, _a(packed), rows, cols, _a(X), batch, _a(Y), nthreads) == 0
        return Y


class Reference:
    """The reference's own kernels (compiled from its sources, unmodified)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        L = C.CDLL(path)
        L.kernel_ctx_create.restype = vp
        L.kernel_ctx_create.argtypes = [i32, i32]
        L.kernel_ctx_init.argtypes = [vp]
        L.kernel_ctx_destroy.argtypes = [vp]
        L.tensor_create_view.restype = vp
        L.tensor_create_view.argtypes = [i32, i32, C.POINTER(i32), vp]
        L.tensor_create.restype = vp
        L.tensor_create.argtypes = [i32, C.POINTER(i32), i32]
        L.tensor_nbytes.restype = C.c_size_t
        L.tensor_nbytes.argtypes = [vp]
        L.tensor_release.argtypes = [vp]
        L.kernel_gemv.argtypes = [vp, vp, vp, vp]
        L.kernel_gemm.argtypes = [vp, vp, vp, vp, i32, i32]
        for n in ("quantized_gemv_q4_0_aligned", "quantized_gemv_q4_0_unaligned",
                  "quantized_gemv_q8_0_aligned", "quantized_gemv_q8_0_unaligned",
                  "quantized_gemv_f32_avx2", "quantized_gemv_bf16_avx2"):
            getattr(L, n).restype = f32
            getattr(L, n).argtypes = [vp, vp, i32, i32]
        L.log_set_level.argtypes = [i32]
        L.log_set_level(40)  # errors only
        self.L = L

    def ctx(self, threads: int = 0):
        c = self.L.kernel_ctx_create(threads, 16)
        assert c and self.L.kernel_ctx_init(c) == 0
        return c

    def view(self, dtype: int, rows: int, cols: int, data: np.ndarray):
        shape = (i32 * 2)(rows, cols)
        return self.L.tensor_create_view(dtype, 2, shape, _a(data))

    def gemv(self, ctx, dtype: int, packed: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        """Reference kernel_gemv (thread pool + AVX2 row kernels).  x is padded."""
        t = self.view(dtype, rows, cols, packed)
        y = np.zeros(rows, dtype=np.float32)
        xx = np.ascontiguousarray(x, dtype=np.float32)
        rc = self.L.kernel_gemv(ctx, _a(y), t, _a(xx))
        self.L.tensor_release(t)
        assert rc == 0, "reference kernel_gemv failed"
        return y


def available_reference() -> bool:
    return os.path.exists(REF_SO)


DECODE_SO = os.path.join(HERE, "_ref", "libdecode_ref.so")


def available_reference_decode() -> bool:
    return os.path.exists(DECODE_SO)


class ReferenceDecode:
    """The reference's Gemma-3 decode (its inference session, layers and
    Q4_0 kernel_gemv, compiled unmodified) driven by oracle/decode_ref.c."""

    def __init__(self, path: str = DECODE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        # Load the reference library first so its log level can be set.
        ref = C.CDLL(REF_SO)
        ref.log_set_level.argtypes = [i32]
        ref.log_set_level(40)  # errors only
        L = C.CDLL(path)
        L.decode_ref_run.restype = i32
        L.decode_ref_run.argtypes = [vp, i32, i32, vp, vp, vp] + [i32] * 9 + [vp, vp, vp, vp, vp]
        self.L = L
        self._ref = ref

    def run(self, cfg, model, n_gen: int | None = None, n_prompt: int | None = None, want_logits: bool = False):
        """(tokens int32 [n_gen], margins f32 [n_gen], logits0 or None,
        prefill seconds, decode seconds) for a model from
        sapphire_b200.workloads.make_decode_model."""
        n_gen = cfg.generate if n_gen is None else n_gen
        prompt = np.ascontiguousarray(model["prompt"][: (n_prompt or cfg.prompt)], dtype=np.int32)
        ptrs = []
        for layer in model["layers"]:
            for name, _, _ in cfg.projections():
                ptrs.append(_a(layer[name]))
        wp = (C.c_void_p * len(ptrs))(*ptrs)
        toks = np.zeros(n_gen, dtype=np.int32)
        margins = np.zeros(n_gen, dtype=np.float32)
        logits = np.zeros(cfg.vocab, dtype=np.float32) if want_logits else None
        tp, td = C.c_double(0), C.c_double(0)
        rc = self.L.decode_ref_run(_a(prompt), len(prompt), n_gen, _a(model["embed"]), C.cast(wp, vp),
                                   _a(model["lm_head"]), cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads,
                                   cfg.head_dim, cfg.vocab, cfg.context, cfg.sliding_window, _a(toks), _a(margins),
                                   _a(logits) if logits is not None else 0, C.addressof(tp), C.addressof(td))
        assert rc == 0, "reference decode failed"
        return toks, margins, logits, tp.value, td.value
