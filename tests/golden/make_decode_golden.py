#!/usr/bin/env python3
"""Golden greedy tokens of the Gemma-3-270M decode workload, from the
reference's own decode (oracle/_ref/libdecode_ref.so, built from the
reference sources by `make -C oracle ref`).

    python tests/golden/make_decode_golden.py

Writes tests/golden/decode_gemma3_270m_seed0.npz: the 64 generated token ids,
their top-1 minus top-2 logit margins, the top 64 logits (ids and values) of
the first generated step, and digests of the generated model so a change of
the generator is detected.  Model and prompt: sapphire_b200.workloads.C3,
make_decode_model(seed 0) with the oracle's Q4_0 quantiser (bit-identical to
the library's GPU quantiser).  Also tests/golden/decode_gqa_tiny_seed3.npz,
the same for sapphire_b200.workloads.GQA_TINY (seed 3).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Oracle, ReferenceDecode  # noqa: E402
from sapphire_b200 import workloads  # noqa: E402


def main():
    write(workloads.C3, 0, "decode_gemma3_270m_seed0.npz")
    # A small grouped-query model (seed 3: its smallest greedy margin, 0.015,
    # is ~5 % of the logit RMS, far above fp32 rounding differences).
    write(workloads.GQA_TINY, 3, "decode_gqa_tiny_seed3.npz")


def write(cfg, seed, name):
    o = Oracle()
    model = workloads.make_decode_model(cfg, lambda a: o.quantize(3, a), seed=seed)
    toks, margins, logits0, tp, td = ReferenceDecode().run(cfg, model, want_logits=True)
    top = np.argsort(-logits0, kind="stable")[:64]
    out = os.path.join(HERE, name)
    np.savez(out, tokens=toks, margins=margins, top_ids=top.astype(np.int32), top_logits=logits0[top],
             logits0_rms=np.float32(np.sqrt(np.mean(logits0.astype(np.float64) ** 2))),
             digest=np.array(workloads.model_digest(model)), prefill_s=np.float64(tp), decode_s=np.float64(td))
    print(f"wrote {out}: tokens {toks[:8]}..., min margin {margins.min():.5f}, "
          f"prompt {tp:.1f} s, generation {td:.1f} s")


if __name__ == "__main__":
    main()
