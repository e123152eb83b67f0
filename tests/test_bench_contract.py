"""The bench's JSON line (reference arm, CPU only): one line with the keys the
round's driver reads, on the smallest configuration (C1, Q4_0 2048 x 640)."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run("--impl", "reference", "--steps", "2", "--warmup", "1", "--config", "q4_0_ffn_up_2048x640")
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 2
    assert d["warmup"] >= 3                     # at least three warm-up steps, whatever was asked
    assert d["value"] > 0 and d["higher_is_better"] is True and d["unit"] == "GB/s"
    assert d["config"]["workload"] == "q4_0_ffn_up_2048x640"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
