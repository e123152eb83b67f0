"""Seeded synthetic inputs of the benchmark configurations.

One documented generator: numpy's PCG64 (`np.random.default_rng(seed)`), draws
taken in the order written below.  Weights are N(0, 0.02) fp32 (quantised by
the library's GPU quantiser where a config asks for Q4_0 / Q8_0), activations
N(0, 1) fp32, ternary codes uniform over {-1, 0, +1} with per-row scales
U(0.01, 0.1).  No dataset is involved.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

# tensor_dtype_t values (include/tensor.h).  Defined here rather than imported
# from the binding so this module loads without libsapphire_cuda.so: the
# benchmark's CPU reference arm imports it by file path and must not map the
# GPU library.
DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_Q4_0, DTYPE_Q8_0, DTYPE_TQ2_0 = range(6)
DTYPE_NAMES = {DTYPE_F32: "F32", DTYPE_BF16: "BF16", DTYPE_F16: "F16", DTYPE_Q4_0: "Q4_0",
               DTYPE_Q8_0: "Q8_0", DTYPE_TQ2_0: "TQ2_0"}


def row_bytes(dtype: int, cols: int) -> int:
    """Bytes of one packed host row: Q4_0 / Q8_0 blocks of 20 / 36 bytes
    (include/kernels.h block structs), TQ2_0 an fp32 row scale and 8 bytes per
    32 trits, F32 / BF16 / F16 dense."""
    nb = (cols + 31) // 32
    if dtype == DTYPE_Q4_0:
        return nb * 20
    if dtype == DTYPE_Q8_0:
        return nb * 36
    if dtype == DTYPE_TQ2_0:
        return 4 + nb * 8
    return cols * (4 if dtype == DTYPE_F32 else 2)


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
# The LM-head shape in the other two formats (the bandwidth target names all
# three on this shape).
C2_Q4 = GemvConfig("q4_0_lm_head_262144x640", DTYPE_Q4_0, 262144, 640)
C2_TQ2 = GemvConfig("tq2_0_lm_head_262144x640", DTYPE_TQ2_0, 262144, 640)
CONFIGS = {c.name: c for c in (C1, C2, C4, C5, C2_Q4, C2_TQ2)}


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


# ------------------------------------------------------------------ decode --
@dataclass(frozen=True)
class DecodeConfig:
    """Gemma-3-270M decode workload (random-init).  Shapes follow the model:
    18 layers, hidden 640, FFN 2048 (GeGLU), 4 query heads / 1 KV head of
    dimension 256, vocabulary 262144.  sliding_window is chosen here (the
    model's own 512; the benchmark names none) so the last generated tokens
    of the local layers attend to a window."""
    name: str = "gemma3_270m_decode"
    layers: int = 18
    hidden: int = 640
    ffn: int = 2048
    heads: int = 4
    kv_heads: int = 1
    head_dim: int = 256
    vocab: int = 262144
    prompt: int = 512
    generate: int = 64
    context: int = 2048
    sliding_window: int = 512
    rope_theta: float = 1.0e6
    rope_local_theta: float = 1.0e4
    query_pre_attn_scalar: float = 256.0
    rms_eps: float = 1e-6

    def is_global(self, layer: int) -> bool:
        return (layer + 1) % 6 == 0

    def projections(self):
        """(name, rows, cols) of one layer's Q4_0 projections, in draw order."""
        q = self.heads * self.head_dim
        kv = self.kv_heads * self.head_dim
        return [("q", q, self.hidden), ("k", kv, self.hidden), ("v", kv, self.hidden),
                ("o", self.hidden, q), ("gate", self.ffn, self.hidden), ("up", self.ffn, self.hidden),
                ("down", self.hidden, self.ffn)]


C3 = DecodeConfig()

# A small grouped-query model for the decode tests: two KV heads shared by
# four query heads, head_dim 64, six layers (layer 5 global), a 32-position
# window - shapes C3 does not exercise.  query_pre_attn_scalar = head_dim, as
# the reference's decode harness sets it.
GQA_TINY = DecodeConfig(name="gqa_tiny", layers=6, hidden=256, ffn=512, heads=4, kv_heads=2, head_dim=64,
                        vocab=4096, prompt=48, generate=24, context=128, sliding_window=32,
                        query_pre_attn_scalar=64.0)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even (finite values)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def make_decode_model(cfg: DecodeConfig, quantize, seed: int = 0):
    """Seeded random-init Gemma-3 weights and prompt.

    Draw order (PCG64 `seed`): prompt ids (cfg.prompt integers in [0, vocab)),
    the embedding table N(0, 0.02) [vocab, hidden] stored as bf16, then for
    each layer q, k, v, o, gate, up, down N(0, 0.02) [rows, cols], then the LM
    head N(0, 0.02) [vocab, hidden].  Projections and LM head are packed Q4_0
    by `quantize(fp32 [rows, cols]) -> packed bytes`.  Norm weights are zero
    (RMSNorm with (1 + w) scaling: scale 1).

    Returns dict(prompt=int32 [prompt], embed=uint16 [vocab*hidden],
    layers=[{name: packed bytes}], lm_head=packed bytes)."""
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg.vocab, size=cfg.prompt, dtype=np.int64).astype(np.int32)
    embed = bf16_bits(normal_weights(rng, cfg.vocab, cfg.hidden)).reshape(-1)
    layers = []
    for _ in range(cfg.layers):
        layers.append({name: quantize(normal_weights(rng, rows, cols)) for name, rows, cols in cfg.projections()})
    lm_head = quantize(normal_weights(rng, cfg.vocab, cfg.hidden))
    return {"prompt": prompt, "embed": embed, "layers": layers, "lm_head": lm_head}


def model_digest(model) -> str:
    """sha256 over the prompt and samples of the model's bytes (embedding head,
    first and last projection, LM head tail): detects a change of the
    generator or the quantiser."""
    h = hashlib.sha256()
    h.update(model["prompt"].tobytes())
    h.update(model["embed"][:1 << 20].tobytes())
    h.update(model["layers"][0]["q"].tobytes())
    h.update(model["layers"][-1]["down"].tobytes())
    h.update(model["lm_head"][-(1 << 20):].tobytes())
    return h.hexdigest()
