"""Device-resident Gemma-3 decoder (include/sapphire_decode.h) from Python.

Mirrors the reference's decode loop (inference_session_create,
inference_forward per token, lm_head, sample_greedy): `Decoder.generate`
orders positions like perform_inference (src/inference/inference.c:238-325).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import SapphireError, addr, lib
from ._lib import Gemma3Config, Gemma3Weights


def config_struct(cfg) -> Gemma3Config:
    """sapphire_gemma3_config_t from a workloads.DecodeConfig."""
    return Gemma3Config(cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab,
                        cfg.context, cfg.sliding_window, cfg.rope_theta, cfg.rope_local_theta,
                        cfg.query_pre_attn_scalar, cfg.rms_eps, 0)


class Decoder:
    """Uploads `model` (workloads.make_decode_model) to the context's GPU."""

    def __init__(self, ctx, cfg, model):
        self.ctx, self.cfg = ctx, cfg
        ptrs = [addr(layer[name]) for layer in model["layers"] for name, _, _ in cfg.projections()]
        self._proj = (C.c_void_p * len(ptrs))(*ptrs)
        w = Gemma3Weights(addr(model["embed"]), addr(model["lm_head"]), None,
                          C.cast(self._proj, C.c_void_p), None)
        c = config_struct(cfg)
        self.handle = lib.sapphire_decoder_create(ctx.handle, C.byref(c), C.byref(w))
        if not self.handle:
            raise SapphireError(f"sapphire_decoder_create failed: {ctx.last_error}")

    @classmethod
    def from_safetensors(cls, ctx, cfg, st):
        """A decoder loaded from a quantized safetensors file
        (sapphire_decoder_create_from_safetensors); `st` is a
        safetensors.SafeTensors, which may be closed afterwards."""
        self = cls.__new__(cls)
        self.ctx, self.cfg = ctx, cfg
        c = config_struct(cfg)
        self.handle = lib.sapphire_decoder_create_from_safetensors(ctx.handle, C.byref(c), st.handle)
        if not self.handle:
            raise SapphireError(f"sapphire_decoder_create_from_safetensors failed: {ctx.last_error}")
        return self

    def generate(self, prompt, n_gen: int):
        """(generated ids int32 [n_gen], top-1 minus top-2 margins f32 [n_gen])."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        ids = np.zeros(max(n_gen, 1), dtype=np.int32)
        margins = np.zeros(max(n_gen, 1), dtype=np.float32)
        rc = lib.sapphire_decoder_generate(self.handle, addr(p), len(p), n_gen, addr(ids), addr(margins))
        if rc != 0:
            raise SapphireError(f"sapphire_decoder_generate failed: {self.ctx.last_error}")
        return ids[:n_gen], margins[:n_gen]

    def last_logits(self) -> np.ndarray:
        out = np.zeros(self.cfg.vocab, dtype=np.float32)
        if lib.sapphire_decoder_last_logits(self.handle, addr(out)) != 0:
            raise SapphireError(f"sapphire_decoder_last_logits failed: {self.ctx.last_error}")
        return out

    def last_times(self):
        """(prompt ms, generation ms) of the last generate, device-timed."""
        a, b = C.c_float(0), C.c_float(0)
        lib.sapphire_decoder_last_times(self.handle, C.byref(a), C.byref(b))
        return a.value, b.value

    @property
    def launches_per_token(self) -> int:
        return lib.sapphire_decoder_launches_per_token(self.handle)

    @property
    def launches_per_prompt_token(self) -> int:
        return lib.sapphire_decoder_launches_per_prompt_token(self.handle)

    def close(self) -> None:
        if self.handle:
            lib.sapphire_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
