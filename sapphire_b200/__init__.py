"""sapphire_b200 - B200-native quantized GEMV hot path of Sapphire.

Python host mirror of the C-ABI in include/kernels.h, include/tensor.h and
include/sapphire_cuda.h.  The names follow the reference's kernel API
(kernel_ctx_create / kernel_gemv / tensor_create_view ...); every product runs
in libsapphire_cuda.so on the GPU.  Buffers may be numpy arrays (host), torch
tensors (host or CUDA) or raw integer addresses.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import (DTYPE_BF16, DTYPE_F16, DTYPE_F32, DTYPE_NAMES, DTYPE_Q4_0, DTYPE_Q8_0,  # noqa: F401
                   DTYPE_TQ2_0, UNIQUE_ID_BYTES, GemmArgs, PARALLEL_FOR_FN)

lib = _lib.load()


class SapphireError(RuntimeError):
    pass


def addr(buf) -> int:
    """Address of a numpy array, torch tensor, ctypes object or int."""
    if buf is None:
        return 0
    if isinstance(buf, int):
        return buf
    if isinstance(buf, np.ndarray):
        return buf.ctypes.data
    if hasattr(buf, "data_ptr"):
        return buf.data_ptr()
    return C.addressof(buf)


def row_bytes(dtype: int, cols: int) -> int:
    """Bytes of one packed row (reference block layout; TQ2_0: scale + blocks)."""
    return int(lib.sapphire_row_bytes(dtype, cols))


class Context:
    """kernel_context_t: one GPU, a stream, resident weights, host workers."""

    def __init__(self, num_threads: int = 0, chunk_size: int = 16, init: bool = True, device: int | None = None):
        self.handle = lib.kernel_ctx_create(num_threads, chunk_size)
        if not self.handle:
            raise SapphireError("kernel_ctx_create failed")
        if device is not None and lib.kernel_ctx_set_device(self.handle, device) != 0:
            msg = self.last_error
            lib.kernel_ctx_destroy(self.handle)
            self.handle = None
            raise SapphireError(f"kernel_ctx_set_device failed: {msg}")
        if init and lib.kernel_ctx_init(self.handle) != 0:
            msg = self.last_error
            lib.kernel_ctx_destroy(self.handle)
            self.handle = None
            raise SapphireError(f"kernel_ctx_init failed: {msg}")

    @property
    def last_error(self) -> str:
        return (lib.kernel_ctx_last_error(self.handle) or b"").decode()

    def check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise SapphireError(f"{what} failed: {self.last_error}")

    def shard(self, rank: int, world: int, unique_id: bytes | None) -> None:
        buf = C.create_string_buffer(unique_id, UNIQUE_ID_BYTES) if unique_id else None
        self.check(lib.kernel_ctx_init_sharded(self.handle, rank, world, buf), "kernel_ctx_init_sharded")

    @property
    def stream(self) -> int:
        return lib.kernel_ctx_get_stream(self.handle) or 0

    @property
    def device(self) -> int:
        return lib.kernel_ctx_get_device(self.handle)

    def synchronize(self) -> None:
        self.check(lib.kernel_ctx_synchronize(self.handle), "kernel_ctx_synchronize")

    def resident_bytes(self) -> int:
        return int(lib.kernel_ctx_resident_bytes(self.handle))

    def close(self) -> None:
        if self.handle:
            lib.kernel_ctx_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_rows(rows: int, rank: int, world: int) -> tuple[int, int]:
    """(row0, nrows) of the rows `rank` of `world` owns (sapphire_shard_rows)."""
    r0, n = C.c_int(0), C.c_int(0)
    if lib.sapphire_shard_rows(rows, rank, world, C.byref(r0), C.byref(n)) != 0:
        raise SapphireError(f"sapphire_shard_rows({rows}, {rank}, {world}) rejected its arguments")
    return r0.value, n.value


def shard_unique_id() -> bytes:
    buf = C.create_string_buffer(UNIQUE_ID_BYTES)
    if lib.kernel_shard_unique_id(buf) != 0:
        raise SapphireError("kernel_shard_unique_id failed")
    return buf.raw


class Tensor:
    """tensor_t view over caller memory (tensor_create_view); keeps `data` alive."""

    def __init__(self, dtype: int, shape, data):
        self.data = data
        self.shape = tuple(int(s) for s in shape)
        arr = (C.c_int * len(self.shape))(*self.shape)
        self.handle = lib.tensor_create_view(dtype, len(self.shape), arr, addr(data))
        if not self.handle:
            raise SapphireError("tensor_create_view failed")
        self.dtype = dtype

    def release(self) -> None:
        if self.handle:
            lib.tensor_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def gemv(ctx: Context | None, A: Tensor, x, y=None):
    """y = A @ x through kernel_gemv (host numpy in/out by default)."""
    rows = A.shape[0]
    if y is None:
        y = np.zeros(rows, dtype=np.float32)
    rc = lib.kernel_gemv(ctx.handle if ctx else None, addr(y), A.handle, addr(x))
    if rc != 0:
        raise SapphireError(f"kernel_gemv failed: {ctx.last_error if ctx else ''}")
    return y


def gemm(ctx: Context, A: Tensor, X, batch: int, Y=None, out_stride: int | None = None):
    """Y[b, :] = A @ X[b, :] through kernel_gemm."""
    rows = A.shape[0]
    if Y is None:
        Y = np.zeros((batch, rows), dtype=np.float32)
    stride = rows if out_stride is None else out_stride
    rc = lib.kernel_gemm(ctx.handle, addr(Y), A.handle, addr(X), batch, stride)
    if rc != 0:
        raise SapphireError(f"kernel_gemm failed: {ctx.last_error}")
    return Y


def quantize(ctx: Context | None, dtype: int, w: np.ndarray, out=None):
    """Pack fp32 [rows, cols] into Q4_0 / Q8_0 blocks on the GPU."""
    rows, cols = w.shape
    if out is None:
        out = np.zeros(rows * row_bytes(dtype, cols), dtype=np.uint8)
    fn = lib.kernel_quantize_q4_0 if dtype == DTYPE_Q4_0 else lib.kernel_quantize_q8_0
    rc = fn(ctx.handle if ctx else None, addr(out), addr(w), rows, cols)
    if rc != 0:
        raise SapphireError("quantize failed")
    return out


def pack_tq2(ctx: Context | None, trits: np.ndarray, scales: np.ndarray, out=None):
    rows, cols = trits.shape
    if out is None:
        out = np.zeros(rows * row_bytes(DTYPE_TQ2_0, cols), dtype=np.uint8)
    rc = lib.kernel_pack_tq2_0(ctx.handle if ctx else None, addr(out), addr(trits), addr(scales), rows, cols)
    if rc != 0:
        raise SapphireError("kernel_pack_tq2_0 failed")
    return out


def dequantize(ctx: Context | None, A: Tensor, out=None):
    rows, cols = A.shape
    if out is None:
        out = np.zeros((rows, cols), dtype=np.float32)
    rc = lib.kernel_dequantize(ctx.handle if ctx else None, addr(out), A.handle)
    if rc != 0:
        raise SapphireError("kernel_dequantize failed")
    return out
