"""Host-side arithmetic of the GEMV kernels' work split (CPU only).

The dense kernel (sapphire_b200/csrc/gemv_pipe.cu) gives warp w the items
[floor(w*T/W), floor((w+1)*T/W)), finds the owner of item i as
ceil((i+1)*W/T) - 1, and sizes the split-tile scratch with
pipe_kmax(T, W, nseg).  These are restated here and checked by brute force:
the owner formula must name the warp whose range holds the item, and no tile
may have more contributing warps than pipe_kmax allows (the scratch slot index
would overflow otherwise).  The streaming kernel of the quantized formats
(sapphire_b200/csrc/gemv_stream.cu: range_begin, unit_owner, stream_kmax)
splits 64-column units over its consumer warps with the same three formulas.
"""
from __future__ import annotations

import itertools


def begin(w, T, W):
    return (w * T) // W


def owner(i, T, W):
    w = ((i + 1) * W + T - 1) // T - 1
    return min(w, W - 1)


def pipe_kmax(T, W, nseg):
    if T <= 0:
        return 1
    if T < W:
        return nseg
    L = T // W
    return min((nseg - 1 + L - 1) // L + 1, nseg)


def check(ntiles, nseg, W):
    T = ntiles * nseg
    # owner(i) is the warp whose range contains i
    for i in range(T):
        w = owner(i, T, W)
        assert begin(w, T, W) <= i < begin(w + 1, T, W), (i, T, W, w)
    kmax = pipe_kmax(T, W, nseg)
    for t in range(ntiles):
        owners = {owner(t * nseg + s, T, W) for s in range(nseg)}
        assert len(owners) <= kmax, (ntiles, nseg, W, len(owners), kmax)


def test_partition_small_exhaustive():
    for ntiles, nseg, W in itertools.product(range(1, 12), range(1, 10), range(1, 40)):
        check(ntiles, nseg, W)


def test_partition_benchmark_shapes():
    W = 148 * 8
    for rows, kchunks in ((262144, 40), (2048, 20), (16384, 256), (10240, 80), (640, 64), (1, 1)):
        ntiles = (rows + 31) // 32
        nseg = (kchunks + 7) // 8
        check(ntiles, nseg, W)


def test_partition_stream_shapes():
    # Units of 64 columns per 32-row tile, 11 (Q8_0 / Q4_0) or 15 (TQ2_0)
    # consumer warps per SM; full weights and the row slices one rank of 2, 4
    # or 8 streams.
    for rows, cols, nc in ((262144, 640, 11), (262144, 640, 15), (16384, 16384, 15), (2048, 640, 11)):
        for world in (1, 2, 4, 8):
            nloc = (rows + world - 1) // world
            check((nloc + 31) // 32, (cols // 32 + 1) // 2, 148 * nc)
