"""Quantized safetensors (include/sapphire_safetensors.h), host side.

The container is the reference's (src/io/safetensors_reader.c:88-250: 8-byte
header length, JSON header, data section); the reader adds the Q4_0 / Q8_0 /
TQ2_0 dtypes the reference's safetensors_create_tensor_ref rejects
(src/io/safetensors_reader.c:405-416).  Files holding only F32 / BF16 / F16
tensors must read the same through both readers.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np
import pytest

from conftest import ROOT

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libsapphire_ref.so")


@pytest.fixture(scope="module")
def st_mod():
    from sapphire_b200 import safetensors
    return safetensors


def _tensors(rng):
    from sapphire_b200.workloads import DTYPE_Q4_0, DTYPE_Q8_0, DTYPE_TQ2_0, row_bytes
    q = lambda dt, r, c: rng.integers(0, 256, size=r * row_bytes(dt, c), dtype=np.uint8)  # noqa: E731
    return {
        "a.f32": ("F32", (3, 5), rng.standard_normal((3, 5)).astype(np.float32)),
        "b.norm.weight": ("BF16", (7,), rng.integers(0, 1 << 16, size=7, dtype=np.uint16)),
        "c.f16": ("F16", (2, 2), rng.standard_normal((2, 2)).astype(np.float16)),
        "d.q4": ("Q4_0", (4, 64), q(DTYPE_Q4_0, 4, 64)),
        "e.q8": ("Q8_0", (3, 100), q(DTYPE_Q8_0, 3, 100)),
        "f.tq2": ("TQ2_0", (2, 300), q(DTYPE_TQ2_0, 2, 300)),
    }


def test_round_trip(st_mod, tmp_path):
    rng = np.random.default_rng(7)
    t = _tensors(rng)
    path = str(tmp_path / "m.safetensors")
    st_mod.save(path, t, metadata={"format": "test"})
    with st_mod.SafeTensors(path) as st:
        assert st.names() == list(t)
        for name, (dtype, shape, data) in t.items():
            got_dtype, got_shape, got = st.info(name)
            assert got_dtype == dtype and got_shape == shape, name
            assert got == np.ascontiguousarray(data).tobytes(), name
        with pytest.raises(KeyError):
            st.tensor("absent")
        # Views are owned by the file: asking twice gives the same tensor.
        assert st.tensor("d.q4") == st.tensor("d.q4")


def test_empty_file(st_mod, tmp_path):
    path = str(tmp_path / "e.safetensors")
    st_mod.save(path, {})
    with st_mod.SafeTensors(path) as st:
        assert st.names() == []


def _raw(path, header: bytes, data: bytes = b"", hlen=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header) if hlen is None else hlen))
        f.write(header)
        f.write(data)


@pytest.mark.parametrize("case", ["missing", "short", "hlen", "json", "dtype", "shape1d", "size", "beyond",
                                  "offsets_reversed", "no_offsets", "overflow", "dim_too_large"])
def test_rejects_bad_files(st_mod, tmp_path, case):
    from sapphire_b200 import SapphireError
    path = str(tmp_path / f"{case}.safetensors")
    ok = {"w": {"dtype": "Q8_0", "shape": [2, 32], "data_offsets": [0, 72]}}
    if case == "short":
        open(path, "wb").write(b"\x01\x02")
    elif case == "hlen":
        _raw(path, b"{}", hlen=1 << 40)
    elif case == "json":
        _raw(path, json.dumps(ok).encode()[:-3], bytes(72))
    elif case == "dtype":
        _raw(path, json.dumps({"w": {"dtype": "Q5_K", "shape": [2, 32], "data_offsets": [0, 72]}}).encode(),
             bytes(72))
    elif case == "shape1d":
        _raw(path, json.dumps({"w": {"dtype": "Q8_0", "shape": [64], "data_offsets": [0, 72]}}).encode(), bytes(72))
    elif case == "size":
        _raw(path, json.dumps({"w": {"dtype": "Q8_0", "shape": [2, 32], "data_offsets": [0, 70]}}).encode(),
             bytes(72))
    elif case == "beyond":
        _raw(path, json.dumps(ok).encode(), bytes(71))
    elif case == "offsets_reversed":
        _raw(path, json.dumps({"w": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}).encode(), bytes(8))
    elif case == "no_offsets":
        _raw(path, json.dumps({"w": {"dtype": "F32", "shape": [1]}}).encode(), bytes(4))
    elif case == "overflow":
        # 2^62 * 2^2 elements: the byte count wraps to 16 in 64 bits.
        _raw(path, json.dumps({"w": {"dtype": "F32", "shape": [2147483647] * 2 + [1073741825, 2],
                                      "data_offsets": [0, 16]}}).encode(), bytes(16))
    elif case == "dim_too_large":
        _raw(path, json.dumps({"w": {"dtype": "F32", "shape": [1 << 31], "data_offsets": [0, 4]}}).encode(), bytes(4))
    with pytest.raises(SapphireError):
        st_mod.SafeTensors(path)


def test_writer_checks_sizes(st_mod, tmp_path):
    with pytest.raises(ValueError):
        st_mod.save(str(tmp_path / "x.safetensors"), {"w": ("Q4_0", (2, 32), bytes(39))})


class _RefMeta(C.Structure):
    # safetensors_tensor_meta_t of the reference (include/safetensors_reader.h:52-59).
    _fields_ = [("name", C.c_char * 256), ("dtype", C.c_int), ("ndim", C.c_int), ("shape", C.c_uint32 * 8),
                ("offset", C.c_uint64), ("size_bytes", C.c_uint64)]


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built here")
def test_reference_reader_agrees_on_dense_files(st_mod, tmp_path):
    """A file of F32 / BF16 / F16 tensors written here reads the same through
    the reference's own reader: names, shapes and the bytes at each offset."""
    ref = C.CDLL(REF_LIB)
    ref.safetensors_open.restype = C.c_void_p
    ref.safetensors_open.argtypes = [C.c_char_p]
    ref.safetensors_tensor_count.argtypes = [C.c_void_p]
    ref.safetensors_get_tensor_by_name.restype = C.POINTER(_RefMeta)
    ref.safetensors_get_tensor_by_name.argtypes = [C.c_void_p, C.c_char_p]
    ref.safetensors_close.argtypes = [C.c_void_p]
    rng = np.random.default_rng(3)
    t = {k: v for k, v in _tensors(rng).items() if v[0] in ("F32", "BF16", "F16")}
    path = str(tmp_path / "dense.safetensors")
    st_mod.save(path, t)
    raw = open(path, "rb").read()
    data0 = 8 + struct.unpack("<Q", raw[:8])[0]
    h = ref.safetensors_open(path.encode())
    assert h
    try:
        assert ref.safetensors_tensor_count(h) == len(t)
        with st_mod.SafeTensors(path) as st:
            for name, (dtype, shape, data) in t.items():
                m = ref.safetensors_get_tensor_by_name(h, name.encode()).contents
                assert m.ndim == len(shape) and tuple(m.shape[:m.ndim]) == shape
                ref_bytes = raw[data0 + m.offset:data0 + m.offset + m.size_bytes]
                assert ref_bytes == st.info(name)[2] == np.ascontiguousarray(data).tobytes()
    finally:
        ref.safetensors_close(h)


def test_decoder_loader_checks_names_and_shapes(st_mod, tmp_path):
    """sapphire_decoder_create_from_safetensors validates the file before it
    touches a GPU: a missing tensor or a wrong shape fails with the tensor's
    name in the context's last error."""
    import dataclasses

    from sapphire_b200 import lib
    from sapphire_b200.decode import config_struct
    from sapphire_b200.workloads import C3, DTYPE_Q4_0, row_bytes
    cfg = dataclasses.replace(C3, layers=1, vocab=64)
    ctx = lib.kernel_ctx_create(1, 0)
    assert ctx
    try:
        c = config_struct(cfg)
        q4 = lambda r, cols: ("Q4_0", (r, cols), bytes(r * row_bytes(DTYPE_Q4_0, cols)))  # noqa: E731
        t = {"model.embed_tokens.weight": ("BF16", (cfg.vocab, cfg.hidden), bytes(cfg.vocab * cfg.hidden * 2)),
             "lm_head.weight": q4(cfg.vocab, cfg.hidden)}
        hf = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
              "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
        for name, rows, cols in cfg.projections():
            if name != "down":
                t[f"model.layers.0.{hf[name]}.weight"] = q4(rows, cols)
        path = str(tmp_path / "partial.safetensors")
        st_mod.save(path, t)
        with st_mod.SafeTensors(path) as st:
            assert not lib.sapphire_decoder_create_from_safetensors(ctx, C.byref(c), st.handle)
            assert b"model.layers.0.mlp.down_proj.weight" in lib.kernel_ctx_last_error(ctx)
        t["model.layers.0.mlp.down_proj.weight"] = q4(cfg.hidden + 32, cfg.ffn)
        st_mod.save(path, t)
        with st_mod.SafeTensors(path) as st:
            assert not lib.sapphire_decoder_create_from_safetensors(ctx, C.byref(c), st.handle)
            assert b"down_proj" in lib.kernel_ctx_last_error(ctx)
        t["model.layers.0.mlp.down_proj.weight"] = q4(cfg.hidden, cfg.ffn)
        t["model.norm.weight"] = ("F16", (cfg.hidden,), bytes(cfg.hidden * 2))
        st_mod.save(path, t)
        with st_mod.SafeTensors(path) as st:
            assert not lib.sapphire_decoder_create_from_safetensors(ctx, C.byref(c), st.handle)
            assert b"model.norm.weight" in lib.kernel_ctx_last_error(ctx)
    finally:
        lib.kernel_ctx_destroy(ctx)


def test_reader_survives_mutated_files(tmp_path):
    """tests/c/fuzz_safetensors.c: the reader's own sources built with
    AddressSanitizer and UndefinedBehaviorSanitizer, fed 20,000 mutated files
    (about 4 s).  Any out-of-bounds access, use after free, leak or overflow
    ends the run with a non-zero status."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = str(tmp_path / "fuzz_safetensors")
    csrc = os.path.join(ROOT, "sapphire_b200", "csrc")
    build = subprocess.run([cc, "-O1", "-g", "-std=c11", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                            "-fno-omit-frame-pointer", "-I", os.path.join(ROOT, "include"),
                            os.path.join(ROOT, "tests", "c", "fuzz_safetensors.c"),
                            os.path.join(csrc, "safetensors.c"), os.path.join(csrc, "tensor.c"),
                            os.path.join(csrc, "log.c"), "-o", exe], capture_output=True, text=True)
    if build.returncode != 0:
        pytest.skip("sanitizer build unavailable: " + build.stderr[-300:])
    env = dict(os.environ, SAPPHIRE_LOG_LEVEL="100")
    run = subprocess.run([exe, "20000", "1", str(tmp_path / "mutated.safetensors")], capture_output=True,
                         text=True, env=env, timeout=300)
    if "LeakSanitizer has encountered a fatal error" in run.stderr:
        pytest.skip("leak checking is not available in this environment")
    assert run.returncode == 0, run.stderr[-3000:]
    assert run.stdout.startswith("iterations 20000 ")
    opened = int(run.stdout.split()[3])
    assert opened > 0          # some mutated files are still valid and get read


@pytest.mark.gpu
def test_gemv_on_file_tensors(st_mod, sp, ctx, oracle, tmp_path):
    """Q4_0 / Q8_0 / TQ2_0 tensors read from a file are views the GEMV takes
    as they are: kernel_gemv on each view matches the oracle on the same bytes."""
    from conftest import GEMV_RTOL, normwise_rel
    from sapphire_b200 import workloads
    rng = np.random.default_rng(11)
    rows, cols = 3000, 704
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
    tscale = rng.uniform(0.01, 0.1, size=rows).astype(np.float32)
    packed = {"q4": (sp.DTYPE_Q4_0, oracle.quantize(sp.DTYPE_Q4_0, w)),
              "q8": (sp.DTYPE_Q8_0, oracle.quantize(sp.DTYPE_Q8_0, w)),
              "tq2": (sp.DTYPE_TQ2_0, oracle.pack_tq2(trits, tscale))}
    path = str(tmp_path / "w.safetensors")
    st_mod.save(path, {k: (sp.DTYPE_NAMES[dt], (rows, cols), b) for k, (dt, b) in packed.items()})
    x = rng.standard_normal(cols, dtype=np.float32)
    with st_mod.SafeTensors(path) as st:
        for name, (dt, b) in packed.items():
            y = np.zeros(rows, dtype=np.float32)
            assert sp.lib.kernel_gemv(ctx.handle, y.ctypes.data, st.tensor(name), x.ctypes.data) == 0
            ref = oracle.gemv(dt, b, rows, cols, workloads.pad_cols(x[None, :], cols), f64=True)[0]
            assert normwise_rel(y, ref) < GEMV_RTOL, name
        # The weights were uploaded from the mapping: release them before the
        # file closes (the context keys device copies by tensor).
        for name in packed:
            sp.lib.kernel_tensor_evict(ctx.handle, st.tensor(name))
