"""Seeded synthetic inputs of the benchmark configurations.

One documented generator: numpy's PCG64 (`np.random.default_rng(seed)`), draws
taken in the order written below.  Weights are N(0, 0.02) fp32 (quantised by
the library's GPU quantiser where a config asks for Q4_0 / Q8_0), activations
N(0, 1) fp32, ternary codes uniform over {-1, 0, +1} with per-row scales
U(0.01, 0.1).  No dataset is involved.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ._lib import DTYPE_Q4_0, DTYPE_Q8_0, DTYPE_TQ2_0


@dataclass(frozen=True)
class GemvConfig:
    name: str
    dtype: int
    rows: int
    cols: int
    batch: int = 1


# The GEMV-shaped configurations (names follow the measurement table of the
# hot-path scope: C1 FFN-up, C2 LM head, C4 ternary, C5 prefill).
C1 = GemvConfig("q4_0_ffn_up_2048x640", DTYPE_Q4_0, 2048, 640)
C2 = GemvConfig("q8_0_lm_head_262144x640", DTYPE_Q8_0, 262144, 640)
C4 = GemvConfig("tq2_0_16384x16384", DTYPE_TQ2_0, 16384, 16384)
C5 = GemvConfig("q4_0_prefill_10240x2560_x2048", DTYPE_Q4_0, 10240, 2560, batch=2048)
CONFIGS = {c.name: c for c in (C1, C2, C4, C5)}


def normal_weights(rng: np.random.Generator, rows: int, cols: int, std: float = 0.02) -> np.ndarray:
    w = rng.standard_normal((rows, cols), dtype=np.float32)
    w *= np.float32(std)
    return w


def activations(rng: np.random.Generator, batch: int, cols: int) -> np.ndarray:
    return rng.standard_normal((batch, cols), dtype=np.float32)


def ternary(rng: np.random.Generator, rows: int, cols: int):
    trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
    scales = rng.uniform(0.01, 0.1, size=rows).astype(np.float32)
    return trits, scales


def make_inputs(cfg: GemvConfig, seed: int = 0):
    """(weight source, x) for a config.  Weight source: fp32 [rows, cols] for
    Q4_0 / Q8_0, (trits int8 [rows, cols], scales fp32 [rows]) for TQ2_0.
    x: fp32 [batch, cols]."""
    rng = np.random.default_rng(seed)
    if cfg.dtype == DTYPE_TQ2_0:
        src = ternary(rng, cfg.rows, cfg.cols)
    else:
        src = normal_weights(rng, cfg.rows, cfg.cols)
    x = activations(rng, cfg.batch, cfg.cols)
    return src, x


def pad_cols(x: np.ndarray, cols: int) -> np.ndarray:
    """Zero-pad the last axis to a multiple of 32 (quantized rows read whole blocks)."""
    padded = ((cols + 31) // 32) * 32
    if x.shape[-1] == padded:
        return np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape[:-1] + (padded,), dtype=np.float32)
    out[..., :x.shape[-1]] = x
    return out
