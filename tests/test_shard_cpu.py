"""Row sharding host logic on CPU (gloo ranks, no GPU).

A sharded context computes the rows sapphire_shard_rows gives its rank, pads
its slice to ceil(rows / world) rows, all-gathers the slices and copies them
out as Y[b][rows] (dispatch.cu, run_product).  These tests run that data path
with gloo in place of NCCL and the oracle's row kernels in place of the GPU,
at world sizes 2 and 3, and check the assembled result against the unsharded
product bit for bit (rows are independent, so sharding changes no arithmetic).
"""
from __future__ import annotations

import multiprocessing as mp
import socket

import numpy as np
import pytest

from conftest import ROOT

Q4_0, Q8_0, TQ2_0 = 3, 4, 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(dtype, rows, cols, batch, seed):
    import sys
    sys.path.insert(0, ROOT)
    from oracle.oracle import Oracle
    o = Oracle()
    rng = np.random.default_rng(seed)
    if dtype == TQ2_0:
        trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
        scales = rng.uniform(0.01, 0.1, size=rows).astype(np.float32)
        packed = o.pack_tq2(trits, scales)
    else:
        packed = o.quantize(dtype, (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
    X = np.zeros((batch, (cols + 31) // 32 * 32), dtype=np.float32)
    X[:, :cols] = rng.standard_normal((batch, cols)).astype(np.float32)
    return o, packed, X


def _rank_main(rank, world, port, dtype, rows, cols, batch, out):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import sapphire_b200 as sp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        o, packed, X = _case(dtype, rows, cols, batch, seed=rows + cols)
        rb = sp.row_bytes(dtype, cols)
        row0, n = sp.shard_rows(rows, rank, world)
        per = (rows + world - 1) // world
        local = np.zeros((batch, per), dtype=np.float32)
        if n:
            local[:, :n] = o.gemv(dtype, packed[row0 * rb:(row0 + n) * rb], n, cols, X, nthreads=2)
        gathered = [torch.zeros((batch, per)) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(local))
        Y = np.full((batch, rows), np.nan, dtype=np.float32)
        for r in range(world):
            r0, nr = sp.shard_rows(rows, r, world)
            Y[:, r0:r0 + nr] = gathered[r].numpy()[:, :nr]
        if rank == 0:
            full = o.gemv(dtype, packed, rows, cols, X, nthreads=2)
            out.put(bool(np.array_equal(Y, full)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("dtype,rows,cols,batch", [
    (Q8_0, 4096, 640, 1),       # LM-head width
    (TQ2_0, 1000, 2048, 1),     # rows not divisible by the world size
    (Q4_0, 2048, 640, 3),       # batched product
    (Q4_0, 5, 64, 2),           # fewer rows than a full slice per rank
])
def test_sharded_assembly_matches_unsharded(world, dtype, rows, cols, batch):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, dtype, rows, cols, batch, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    assert out.get(timeout=5) is True


@pytest.mark.parametrize("rows", [0, 1, 5, 2048, 10240, 16384, 262144, 262147])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_tile_the_weight(sp, rows, world):
    spans = [sp.shard_rows(rows, r, world) for r in range(world)]
    pos = 0
    for r0, n in spans:
        assert n >= 0
        if n:
            assert r0 == pos
            pos += n
    assert pos == rows
    per = (rows + world - 1) // world
    assert all(n <= per for _, n in spans)


def test_shard_rows_rejects_bad_arguments(sp):
    for args in [(10, 2, 2), (10, -1, 2), (10, 0, 0), (-1, 0, 1)]:
        with pytest.raises(sp.SapphireError):
            sp.shard_rows(*args)
