"""The numerators of the bench's roofline fractions (CPU only): algorithmic
bytes per GEMV, FLOP per prefill product and bytes per decoded token, pinned
to the per-unit figures the workloads are specified with.  A drift here would
silently rescale every `roofline.frac` the bench reports."""
from __future__ import annotations

import sys

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402

WL = bench.WL


def _bytes(cfg):
    return bench.algorithmic_bytes(cfg.dtype, cfg.rows, cfg.cols)


def test_gemv_bytes_per_product():
    # Q4_0 FFN up 2048 x 640: 819,200 B of blocks + 2,560 B of x + 8,192 B of y.
    assert _bytes(WL.C1) == 829_952
    # Q8_0 LM head 262144 x 640: 188,743,680 + 2,560 + 1,048,576.
    assert _bytes(WL.C2) == 189_794_816
    # Q4_0 on the LM-head shape: 104,857,600 + 2,560 + 1,048,576.
    assert _bytes(WL.C2_Q4) == 105_908_736
    # Ternary 16384 x 16384 at 2 bits per trit: 67,108,864 + 65,536 (row
    # scales) + 65,536 (x) + 65,536 (y).
    assert _bytes(WL.C4) == 67_305_472


def test_row_bytes_follow_the_block_formats():
    # 20-byte Q4_0 and 36-byte Q8_0 blocks per 32 columns; a ternary row is a
    # 4-byte scale and 8 bytes per 32 columns.
    for cols in (32, 640, 2560, 16384):
        nb = cols // 32
        assert WL.row_bytes(WL.DTYPE_Q4_0, cols) == 20 * nb
        assert WL.row_bytes(WL.DTYPE_Q8_0, cols) == 36 * nb
        assert WL.row_bytes(WL.DTYPE_TQ2_0, cols) == 4 + 8 * nb
    # A ragged last block still takes a whole block.
    assert WL.row_bytes(WL.DTYPE_Q4_0, 33) == 40


def test_prefill_flop_count():
    # 2 * tokens * rows * cols for 2048 tokens through the 10240 x 2560 weight.
    assert bench.prefill_flops(WL.C5) == 107_374_182_400
    assert bench.prefill_flops(WL.C5, tokens=1) == 2 * 10240 * 2560


def test_decode_bytes_per_token():
    cfg = WL.C3
    proj = sum(rows * WL.row_bytes(WL.DTYPE_Q4_0, cols) for _, rows, cols in cfg.projections())
    assert proj * cfg.layers == 62_668_800          # the 18 layers' Q4_0 projections
    assert cfg.vocab * WL.row_bytes(WL.DTYPE_Q4_0, cfg.hidden) == 104_857_600   # the LM head
    # About 187 MB per generated token over the 64 greedy steps after the
    # 512-token prompt (weights + embedding row + the KV rows read and written).
    first = bench.decode_bytes_per_token(cfg, cfg.prompt - 1)
    last = bench.decode_bytes_per_token(cfg, cfg.prompt + cfg.generate - 1)
    assert 186e6 < first < last < 188e6
    # Only the global layers read more keys as the position grows.
    n_global = sum(1 for layer in range(cfg.layers) if cfg.is_global(layer))
    kv_row = cfg.kv_heads * cfg.head_dim * 4
    assert last - first == 2 * cfg.generate * kv_row * n_global
