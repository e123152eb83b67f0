"""Device-resident Gemma-3-270M decode against the reference's own decode.

tests/golden/decode_gemma3_270m_seed0.npz holds the greedy ids the reference
produced (its inference session, layers and Q4_0 kernel_gemv, run by
oracle/decode_ref.c; tests/golden/make_decode_golden.py) for the seeded
random-init model of sapphire_b200.workloads.C3: a 512-token prompt, then 64
greedy tokens.  The GPU decoder must produce the same 64 ids.
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

Q4_0 = 3


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "decode_gemma3_270m_seed0.npz"))


@pytest.fixture(scope="module")
def decoder(sp, ctx, golden):
    from sapphire_b200 import workloads
    from sapphire_b200.decode import Decoder
    cfg = workloads.C3
    model = workloads.make_decode_model(cfg, lambda a: sp.quantize(ctx, Q4_0, a), seed=0)
    # Same model bytes as the reference run (GPU quantiser == oracle quantiser).
    assert workloads.model_digest(model) == str(golden["digest"])
    dec = Decoder(ctx, cfg, model)
    yield cfg, model, dec
    dec.close()


def test_greedy_tokens_match_reference(decoder, golden):
    cfg, model, dec = decoder
    ids, margins = dec.generate(model["prompt"], cfg.generate)
    ref = golden["tokens"]
    mismatch = np.nonzero(ids != ref)[0]
    assert mismatch.size == 0, (
        f"first mismatch at step {mismatch[0]}: got {ids[mismatch[0]]}, reference {ref[mismatch[0]]}, "
        f"reference margin {golden['margins'][mismatch[0]]:.5f}")
    # The top-1 minus top-2 margins agree with the reference's to rounding.
    assert np.max(np.abs(margins - golden["margins"])) < 2e-3


def test_first_step_logits(decoder, golden):
    cfg, model, dec = decoder
    ids, _ = dec.generate(model["prompt"], 1)
    assert ids[0] == golden["tokens"][0]
    logits = dec.last_logits()
    top = golden["top_ids"]
    # The reference's 64 largest logits, value by value.
    err = np.max(np.abs(logits[top] - golden["top_logits"]))
    assert err < 2e-3 * float(golden["logits0_rms"]) * 10, err
    rms = float(np.sqrt(np.mean(logits.astype(np.float64) ** 2)))
    assert abs(rms - float(golden["logits0_rms"])) < 1e-3 * rms


def test_generate_is_repeatable(decoder):
    cfg, model, dec = decoder
    a, _ = dec.generate(model["prompt"][:40], 8)
    b, _ = dec.generate(model["prompt"][:40], 8)
    assert np.array_equal(a, b)
    assert dec.launches_per_token > 0


def test_generate_rejects_bad_input(sp, decoder):
    cfg, model, dec = decoder
    with pytest.raises(sp.SapphireError):
        dec.generate(np.array([cfg.vocab], dtype=np.int32), 1)
    with pytest.raises(sp.SapphireError):
        dec.generate(model["prompt"], cfg.context)


def test_decoder_from_quantized_safetensors(sp, ctx, decoder, golden, tmp_path):
    """The same model written as a quantized safetensors file (Q4_0
    projections and LM head under the reference's tensor names) loads through
    sapphire_decoder_create_from_safetensors and decodes the reference's ids."""
    from sapphire_b200 import safetensors
    from sapphire_b200.decode import Decoder
    cfg, model, _ = decoder
    path = str(tmp_path / "gemma3_q4_0.safetensors")
    safetensors.save_decode_model(path, cfg, model)
    with safetensors.SafeTensors(path) as st:
        assert st.info("lm_head.weight")[:2] == ("Q4_0", (cfg.vocab, cfg.hidden))
        dec = Decoder.from_safetensors(ctx, cfg, st)
    # The file is closed: everything the decoder uses lives on the GPU.
    os.remove(path)
    try:
        ids, _ = dec.generate(model["prompt"], cfg.generate)
        assert np.array_equal(ids, golden["tokens"])
    finally:
        dec.close()


def test_from_safetensors_rejects_wrong_dtype(sp, ctx, decoder, tmp_path):
    """An LM head stored as BF16 (the reference's tied-embedding layout) is not
    a quantized product here: creation fails with the tensor named."""
    from sapphire_b200 import safetensors
    from sapphire_b200.decode import Decoder
    cfg, model, _ = decoder
    small = dataclasses.replace(cfg, layers=1)
    path = str(tmp_path / "bad.safetensors")
    t = {"model.embed_tokens.weight": ("BF16", (cfg.vocab, cfg.hidden), model["embed"]),
         "lm_head.weight": ("BF16", (cfg.vocab, cfg.hidden), model["embed"])}
    hf = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
          "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
    for name, rows, cols in small.projections():
        t[f"model.layers.0.{hf[name]}.weight"] = ("Q4_0", (rows, cols), model["layers"][0][name])
    safetensors.save(path, t)
    with safetensors.SafeTensors(path) as st:
        with pytest.raises(sp.SapphireError, match="lm_head.weight"):
            Decoder.from_safetensors(ctx, small, st)


def test_stage_per_kernel_path_matches_reference(sp, ctx, decoder, golden, monkeypatch):
    """The one-kernel-per-stage step (SAPPHIRE_DECODE_PERSISTENT=0 at
    creation) gives the reference's ids as well."""
    from sapphire_b200.decode import Decoder
    cfg, model, _ = decoder
    monkeypatch.setenv("SAPPHIRE_DECODE_PERSISTENT", "0")
    dec = Decoder(ctx, cfg, model)
    try:
        assert dec.launches_per_token > 10      # one kernel per stage
        ids, _ = dec.generate(model["prompt"], cfg.generate)
        assert np.array_equal(ids, golden["tokens"])
    finally:
        dec.close()


def test_persistent_step_reports_an_expired_wait(sp, ctx, decoder, golden):
    """A persistent step in which one block never writes its output (a test
    hook: nothing sets the words the others wait for) gives up after its
    bounded wait: creation fails with the expiry reported, no GPU fault, and a
    decoder created afterwards still decodes the reference's ids."""
    from sapphire_b200.decode import Decoder
    cfg, model, dec = decoder
    assert dec.launches_per_token == 3          # persistent step + LM head + argmax
    assert dec.launches_per_prompt_token == 1
    prev = sp.lib.sapphire_test_decode_stall(1)
    try:
        with pytest.raises(sp.SapphireError, match="gave up waiting"):
            Decoder(ctx, cfg, model)
    finally:
        sp.lib.sapphire_test_decode_stall(prev)
    ok = Decoder(ctx, cfg, model)
    try:
        ids, _ = ok.generate(model["prompt"][:64], 8)
        ref, _ = dec.generate(model["prompt"][:64], 8)
        assert np.array_equal(ids, ref)
    finally:
        ok.close()


@pytest.mark.parametrize("persistent", ["1", "0"])
def test_grouped_query_model_matches_reference(sp, ctx, monkeypatch, persistent):
    """A small grouped-query model (two KV heads for four query heads,
    head_dim 64, a global and five local layers, window 32) decodes the
    reference decode's ids through both step implementations
    (tests/golden/decode_gqa_tiny_seed3.npz, tests/golden/make_decode_golden.py)."""
    from sapphire_b200 import workloads
    from sapphire_b200.decode import Decoder
    golden = np.load(os.path.join(GOLDEN, "decode_gqa_tiny_seed3.npz"))
    cfg = workloads.GQA_TINY
    model = workloads.make_decode_model(cfg, lambda a: sp.quantize(ctx, Q4_0, a), seed=3)
    assert workloads.model_digest(model) == str(golden["digest"])
    monkeypatch.setenv("SAPPHIRE_DECODE_PERSISTENT", persistent)
    dec = Decoder(ctx, cfg, model)
    try:
        # 3 launches per generated token for the persistent step, 5 per layer otherwise.
        assert (dec.launches_per_token == 3) == (persistent == "1")
        ids, margins = dec.generate(model["prompt"], cfg.generate)
        assert np.array_equal(ids, golden["tokens"]), (ids, golden["tokens"])
        assert np.max(np.abs(margins - golden["margins"])) < 1e-3
    finally:
        dec.close()


def test_long_prompt_paths_agree(sp, ctx, decoder, monkeypatch):
    """A 1900-token prompt (global layers attend to every position: up to 56
    keys per split over 37 splits per head) gives the same logits through the
    persistent step and through the per-stage path, to fp32 rounding."""
    from sapphire_b200.decode import Decoder
    cfg, model, dec = decoder
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, size=1900).astype(np.int32)
    ids_p, _ = dec.generate(prompt, 1)
    logits_p = dec.last_logits()
    monkeypatch.setenv("SAPPHIRE_DECODE_PERSISTENT", "0")
    ref = Decoder(ctx, cfg, model)
    try:
        ids_s, _ = ref.generate(prompt, 1)
        logits_s = ref.last_logits()
    finally:
        ref.close()
    err = float(np.max(np.abs(logits_p - logits_s)) / np.max(np.abs(logits_s)))
    assert err < 1e-4, err
    top2 = np.sort(logits_s)[-2:]
    if top2[1] - top2[0] > 1e-3:
        assert ids_p[0] == ids_s[0]
