"""Host-side arithmetic of the pipelined GEMV's work split (CPU only).

The kernel (sapphire_b200/csrc/gemv_pipe.cu) gives warp w the items
[floor(w*T/W), floor((w+1)*T/W)), finds the owner of item i as
ceil((i+1)*W/T) - 1, and sizes the split-tile scratch with
pipe_kmax(T, W, nseg).  These are restated here and checked by brute force:
the owner formula must name the warp whose range holds the item, and no tile
may have more contributing warps than pipe_kmax allows (the scratch slot index
would overflow otherwise).
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
