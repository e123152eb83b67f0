"""Row-sharded products on 2 GPUs: one process per GPU, NCCL all-gather inside
the library.  Skipped when fewer than two GPUs are visible.

Each rank binds its context to its GPU, joins the NCCL group (unique id from
rank 0, passed over a gloo group), and runs the same calls an unsharded
context would: every rank receives the full result, which must match the
oracle (the reference row kernels) within the GEMV bar and be the same bytes
on both ranks.  Batch-1 products of the streaming GEMV are gathered over peer
memory inside the GEMV (epoch-tagged NVLink stores); batched products over
NCCL.  Then the Gemma-3-270M decode runs with its LM head row-sharded: each
rank reduces its logits slice to (value, index) pairs exchanged over peer
memory, and both ranks must emit the reference decode's 64 greedy ids (twice:
the exchange's epochs carry over between requests) with the same margins;
the gathered logits (the parity mode) must peak at the last id.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from conftest import GEMV_RTOL, ROOT

pytestmark = pytest.mark.gpu

Q4_0, Q8_0, TQ2_0 = 3, 4, 5

CASES = [
    # (dtype, rows, cols, batch)
    (Q8_0, 32768, 640, 1),      # LM-head width, pipelined GEMV per rank, gathered over peer memory
    (Q8_0, 3001, 640, 1),       # ragged rows: the last rank holds one row fewer
    (TQ2_0, 4096, 4096, 1),     # ternary
    (Q4_0, 3000, 640, 3),       # batched, per-token GEMV; rows not divisible by 2
    (Q4_0, 2048, 2560, 64),     # tensor-core prefill product per rank
]


def _bf16_round(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _case(o, dtype, rows, cols, batch, seed):
    rng = np.random.default_rng(seed)
    if dtype == TQ2_0:
        trits = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
        scales = rng.uniform(0.01, 0.1, size=rows).astype(np.float32)
        packed = o.pack_tq2(trits, scales)
    else:
        packed = o.quantize(dtype, (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
    X = np.zeros((batch, (cols + 31) // 32 * 32), dtype=np.float32)
    X[:, :cols] = rng.standard_normal((batch, cols)).astype(np.float32)
    return packed, X


def _rank_main(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import sapphire_b200 as sp
    from oracle.oracle import Oracle

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    ctx = None
    try:
        ctx = sp.Context(num_threads=1, device=rank)
        ids = [sp.shard_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        ctx.shard(rank, world, ids[0])
        o = Oracle()
        results = []
        for i, (dtype, rows, cols, batch) in enumerate(CASES):
            packed, X = _case(o, dtype, rows, cols, batch, seed=100 + i)
            A = sp.Tensor(dtype, (rows, cols), packed)
            Y = sp.gemm(ctx, A, np.ascontiguousarray(X[:, :cols]), batch)
            # Repeated products alternate the two gather buffers.
            for _ in range(3):
                Y2 = sp.gemm(ctx, A, np.ascontiguousarray(X[:, :cols]), batch)
                assert np.array_equal(Y, Y2)
            A.release()
            mine = torch.from_numpy(Y.copy())
            other = [torch.zeros_like(mine) for _ in range(world)]
            dist.all_gather(other, mine)
            same = all(torch.equal(other[0], t) for t in other)
            if rank == 0:
                Xr = _bf16_round(X) if (dtype == Q4_0 and batch >= 16) else X
                ref = o.gemv(dtype, packed, rows, cols, Xr)
                err = float(np.max(np.abs(Y - ref)) / np.max(np.abs(ref)))
                results.append((dtype, rows, batch, same, err))
        # Gemma-3-270M decode with the LM head row-sharded: every rank runs the
        # layers, computes its slice of the logits and exchanges (value, index)
        # pairs; both ranks must produce the reference decode's greedy ids.
        from sapphire_b200 import workloads
        from sapphire_b200.decode import Decoder
        cfg = workloads.C3
        model = workloads.make_decode_model(cfg, lambda a: sp.quantize(ctx, 3, a), seed=0)
        dec = Decoder(ctx, cfg, model)
        ids, margins = dec.generate(model["prompt"], cfg.generate)
        ids2, _ = dec.generate(model["prompt"], cfg.generate)          # a second request, epochs continue
        logits = dec.last_logits()                                    # collective: gathered slices
        dec.close()
        golden = np.load(os.path.join(ROOT, "tests", "golden", "decode_gemma3_270m_seed0.npz"))
        dec_ok = bool(np.array_equal(ids, golden["tokens"]) and np.array_equal(ids2, ids))
        top = int(np.argmax(logits))
        mine_ids = torch.from_numpy(ids.astype(np.int64))
        all_ids = [torch.zeros_like(mine_ids) for _ in range(world)]
        dist.all_gather(all_ids, mine_ids)
        dec_same = all(torch.equal(all_ids[0], t) for t in all_ids)
        if rank == 0:
            results.append(("decode", dec_ok, dec_same, top == int(ids[-1]),
                            float(np.max(np.abs(margins - golden["margins"])))))
            out.put(results)
    finally:
        if ctx is not None:
            ctx.close()
        dist.destroy_process_group()


def test_sharded_products_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    results = out.get(timeout=10)
    assert len(results) == len(CASES) + 1
    for dtype, rows, batch, same, err in results[:-1]:
        assert same, (dtype, rows, batch)
        assert err < GEMV_RTOL, (dtype, rows, batch, err)
    _, dec_ok, dec_same, last_is_argmax, margin_err = results[-1]
    assert dec_ok and dec_same and last_is_argmax, results[-1]
    assert margin_err < 2e-3, margin_err
