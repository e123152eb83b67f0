"""Device-resident Gemma-3-270M decode against the reference's own decode.

tests/golden/decode_gemma3_270m_seed0.npz holds the greedy ids the reference
produced (its inference session, layers and Q4_0 kernel_gemv, run by
oracle/decode_ref.c; tests/golden/make_decode_golden.py) for the seeded
random-init model of sapphire_b200.workloads.C3: a 512-token prompt, then 64
greedy tokens.  The GPU decoder must produce the same 64 ids.
"""
from __future__ import annotations

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
