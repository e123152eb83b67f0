"""The reference's own C tests and end-to-end bench, compiled unchanged and
linked against libsapphire_cuda.so (tests/c/Makefile): the drop-in check of
the C-ABI with the reference's callers rather than ctypes.

* test_tensor (reference src/test/test_tensor.c) exercises only the host
  tensor API, so it runs here on the CPU, once as built by the Makefile and
  once built from source with sanitizers;
* test_dispatch (src/test/test_dispatch.c: the Q4_0 row kernels, aligned and
  unaligned, within 1e-4 of each other) and test_tensor_gemv
  (src/test/test_tensor_gemv.c: kernel_gemv / _add / _batch / _tensor and the
  NULL-context rules) run on the GPU and must exit 0 with no failed case;
* bench_end_to_end (src/test/bench/bench_sapphire_end_to_end.c) runs
  kernel_gemv on its deterministic Q4_0 / Q8_0 patterns for five shapes and
  several context thread counts; every printed sum= must match the sum the
  reference's own CPU kernels produced (tests/golden/patterns.npz, generated
  by tests/golden/make_golden.py) within 1e-4 relative.

The binaries are built by __graft_entry__.build() (or `make -C tests/c`) where
the reference checkout exists; elsewhere the prebuilt ones travel with the
tree.  Missing binaries skip.
"""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

BUILD = os.path.join(ROOT, "tests", "c", "_build")


def _bin(name: str) -> str:
    path = os.path.join(BUILD, name)
    if not os.path.exists(path):
        pytest.skip(f"{path} not built (make -C tests/c needs the reference checkout)")
    return path


def _run(name: str, timeout: float = 300.0) -> subprocess.CompletedProcess:
    return subprocess.run([_bin(name)], capture_output=True, text=True, timeout=timeout)


def test_reference_tensor_api_test_passes():
    r = _run("test_tensor")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    m = re.search(r"(\d+) passed, (\d+) failed", r.stdout)
    assert m and int(m.group(2)) == 0 and int(m.group(1)) > 0, r.stdout[-2000:]


def test_reference_tensor_api_test_under_sanitizers(tmp_path):
    """The reference's test_tensor.c against this library's tensor.c, built
    from source with AddressSanitizer and UndefinedBehaviorSanitizer: every
    case passes with no out-of-bounds access, use after free or leak."""
    import shutil
    ref = os.environ.get("SAPPHIRE_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
    src = os.path.join(ref, "src", "test", "test_tensor.c")
    cc = shutil.which("gcc") or shutil.which("cc")
    if not os.path.exists(src) or cc is None:
        pytest.skip("needs the reference checkout and a C compiler")
    exe = str(tmp_path / "test_tensor_asan")
    csrc = os.path.join(ROOT, "sapphire_b200", "csrc")
    build = subprocess.run([cc, "-O1", "-g", "-std=c11", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                            "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ref, "include"), src,
                            os.path.join(csrc, "tensor.c"), os.path.join(csrc, "log.c"),
                            os.path.join(ROOT, "tests", "c", "tensor_hooks.c"), "-o", exe, "-lm"],
                           capture_output=True, text=True)
    if build.returncode != 0:
        pytest.skip("sanitizer build unavailable: " + build.stderr[-300:])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    if "LeakSanitizer has encountered a fatal error" in r.stderr:
        pytest.skip("leak checking is not available in this environment")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    m = re.search(r"(\d+) passed, (\d+) failed", r.stdout)
    assert m and int(m.group(2)) == 0 and int(m.group(1)) > 0, r.stdout[-2000:]


@pytest.mark.gpu
def test_reference_dispatch_test_passes():
    r = _run("test_dispatch")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "aligned=" in r.stdout


@pytest.mark.gpu
def test_reference_tensor_gemv_test_passes():
    r = _run("test_tensor_gemv")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    m = re.search(r"(\d+) passed, (\d+) failed", r.stdout)
    assert m and int(m.group(2)) == 0 and int(m.group(1)) > 0, r.stdout[-3000:]


@pytest.mark.gpu
def test_reference_end_to_end_bench_sums_match_reference():
    r = _run("bench_end_to_end", timeout=600.0)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    golden = np.load(os.path.join(GOLDEN, "patterns.npz"))
    # Sections per configuration, in the bench's order; each holds Q4 and Q8
    # lines for several context thread counts.
    sections = re.split(r"=== CONFIG: rows=(\d+) blocks_per_row=(\d+) ===", r.stdout)[1:]
    assert len(sections) == 3 * 5, r.stdout[-2000:]
    checked = 0
    for i in range(5):
        rows, bpr, body = int(sections[3 * i]), int(sections[3 * i + 1]), sections[3 * i + 2]
        assert tuple(int(v) for v in golden[f"e2e_{i}_shape"]) == (rows, bpr * 32)
        for line in body.splitlines():
            m = re.match(r"\s*(Q4|Q8)\b.*sum=\s*(\S+)\s+rc=\s*(-?\d+)", line)
            if not m:
                continue
            assert int(m.group(3)) == 0, line
            ref = float(golden[f"e2e{m.group(1).lower()}_{i}_sum"])
            got = float(m.group(2))
            assert abs(got - ref) <= 1e-4 * max(1.0, abs(ref)), (line, ref)
            checked += 1
    assert checked >= 20, r.stdout[-2000:]
