"""The committed decode golden files are what the reference's own decode
produces (CPU only).

tests/golden/decode_gemma3_270m_seed0.npz and decode_gqa_tiny_seed3.npz were
written by tests/golden/make_decode_golden.py through
oracle/_ref/libdecode_ref.so (the reference's inference session, layers and
Q4_0 kernel_gemv, compiled from its sources).  These tests rebuild each model,
check it hashes to the digest recorded in the file, run the reference decode
again and require the same greedy ids, so the fixtures the GPU decode is held
to stay pinned to the reference rather than to a file.  The Gemma-3-270M case
takes about a minute (40 s to build the random-init model, 20 s of reference
decode on the host's threads).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)
from oracle.oracle import Oracle, ReferenceDecode, available_reference_decode  # noqa: E402
from sapphire_b200 import workloads  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden")
CASES = [(workloads.GQA_TINY, 3, "decode_gqa_tiny_seed3.npz"), (workloads.C3, 0, "decode_gemma3_270m_seed0.npz")]


@pytest.mark.skipif(not available_reference_decode(), reason="oracle/_ref not built (make -C oracle ref)")
@pytest.mark.parametrize("cfg,seed,name", CASES, ids=[c[0].name for c in CASES])
def test_golden_is_the_reference_decode(cfg, seed, name):
    golden = np.load(os.path.join(GOLDEN, name))
    o = Oracle()
    model = workloads.make_decode_model(cfg, lambda a: o.quantize(3, a), seed=seed)
    assert workloads.model_digest(model) == str(golden["digest"])
    toks, margins, logits0, _, _ = ReferenceDecode().run(cfg, model, want_logits=True)
    np.testing.assert_array_equal(toks, golden["tokens"])
    # Same library, same inputs: the logits agree to rounding of the thread
    # split at most.
    np.testing.assert_allclose(margins, golden["margins"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(logits0[golden["top_ids"]], golden["top_logits"], rtol=0, atol=1e-5)
