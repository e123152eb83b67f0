"""Safetensors files with quantized weights (include/sapphire_safetensors.h).

`save` writes the container the reference reads (an 8-byte little-endian
header length, a JSON header, the data) with this library's added dtypes
"Q4_0", "Q8_0" and "TQ2_0" (packed rows, logical [rows, cols] shape);
`SafeTensors` maps a file through the C-ABI and hands out zero-copy tensor
views; `save_decode_model` writes a Gemma-3 model under the reference's
tensor names (src/loader/gemma3_map.c) so `Decoder.from_safetensors` can load
it.
"""
from __future__ import annotations

import ctypes as C
import json
import struct

import numpy as np

from . import SapphireError, lib
from .workloads import DTYPE_NAMES, row_bytes

_NUMPY_DTYPES = {"F32": np.float32, "BF16": np.uint16, "F16": np.float16}
_QUANTIZED = {"Q4_0": 3, "Q8_0": 4, "TQ2_0": 5}


def _payload_bytes(dtype: str, shape) -> int:
    if dtype in _QUANTIZED:
        rows, cols = shape
        return rows * row_bytes(_QUANTIZED[dtype], cols)
    n = int(np.prod(shape)) if len(shape) else 1
    return n * (4 if dtype == "F32" else 2)


def save(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """tensors: name -> (dtype string, shape, bytes-like or numpy array).
    Quantized payloads are packed rows (rows * row_bytes(cols) bytes)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, shape, data) in tensors.items():
        raw = np.ascontiguousarray(data).reshape(-1).view(np.uint8).tobytes() if isinstance(data, np.ndarray) \
            else bytes(data)
        want = _payload_bytes(dtype, shape)
        if len(raw) != want:
            raise ValueError(f"{name}: {len(raw)} bytes for {dtype} {tuple(shape)}, expected {want}")
        header[name] = {"dtype": dtype, "shape": [int(v) for v in shape], "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


class SafeTensors:
    """A mapped file (sapphire_safetensors_open); tensors are views owned by it."""

    def __init__(self, path: str):
        self.handle = lib.sapphire_safetensors_open(path.encode())
        if not self.handle:
            raise SapphireError(f"sapphire_safetensors_open failed for {path}")

    def names(self) -> list[str]:
        n = lib.sapphire_safetensors_count(self.handle)
        return [lib.sapphire_safetensors_name(self.handle, i).decode() for i in range(n)]

    def tensor(self, name: str) -> int:
        """tensor_t handle (an int) of a view into the mapping; do not release it."""
        t = lib.sapphire_safetensors_tensor(self.handle, name.encode())
        if not t:
            raise KeyError(name)
        return t

    def info(self, name: str):
        """(dtype name, shape, bytes) of a tensor, read through the tensor API."""
        t = self.tensor(name)
        nd = lib.tensor_ndim(t)
        shape = tuple(lib.tensor_shape(t)[i] for i in range(nd))
        dtype = DTYPE_NAMES[lib.tensor_dtype(t)]
        n = _payload_bytes(dtype, shape)
        data = C.string_at(lib.tensor_data(t), n)
        return dtype, shape, data

    def close(self) -> None:
        if self.handle:
            lib.sapphire_safetensors_close(self.handle)
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


def save_decode_model(path: str, cfg, model) -> None:
    """A model from workloads.make_decode_model under the reference's tensor
    names: BF16 embedding, Q4_0 projections and LM head, zero norms omitted
    (absent norms load as zeros)."""
    t = {"model.embed_tokens.weight": ("BF16", (cfg.vocab, cfg.hidden), model["embed"])}
    hf = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
          "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
    for layer, weights in enumerate(model["layers"]):
        for name, rows, cols in cfg.projections():
            t[f"model.layers.{layer}.{hf[name]}.weight"] = ("Q4_0", (rows, cols), weights[name])
    t["lm_head.weight"] = ("Q4_0", (cfg.vocab, cfg.hidden), model["lm_head"])
    save(path, t, metadata={"format": "sapphire quantized", "model": "gemma3"})
