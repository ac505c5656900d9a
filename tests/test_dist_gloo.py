"""The sharded path's host logic on CPU ranks (gloo, world_size 2).

Each rank takes its rows with the library's own partition rule
(m3g_shard_plan, pure host code), computes them with the CPU oracle (the
stand-in for the local GPU GEMV), and the ranks all-gather the slices over
gloo exactly as the GPU path all-gathers over NCCL.  The concatenation must
equal the unsharded result row for row.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CASES = [
    (12, 512, 96),    # divisible
    (14, 256, 37),    # uneven: the last rank holds fewer rows
    (8, 64, 3),       # fewer rows than a full split
    (2, 96, 1),       # one row: rank 1 holds none
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from m3_avm_b200 import sharded, synth
        from oracle import oracle as O

        out = []
        for dtype, in_dim, out_dim in CASES:
            raw = synth.weights(dtype, in_dim, out_dim, seed=in_dim + out_dim)
            x = synth.activations(in_dim, seed=3)
            row0, rows, rpr, b0, blen = sharded.shard_plan(dtype, in_dim, out_dim, world, rank)
            local = np.zeros(rpr, np.float32)
            if rows:
                local[:rows] = O.matvec_quant(x, raw[b0:b0 + blen], dtype, in_dim, rows, threads=1)
            parts = [torch.zeros(rpr) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(local))
            y = torch.cat(parts).numpy()[:out_dim]
            out.append((row0, rows, y))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_row_sharding_all_gather_equals_unsharded():
    from m3_avm_b200 import synth
    from oracle import oracle as O

    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True, start_method="spawn")
    for ci, (dtype, in_dim, out_dim) in enumerate(CASES):
        raw = synth.weights(dtype, in_dim, out_dim, seed=in_dim + out_dim)
        x = synth.activations(in_dim, seed=3)
        full = O.matvec_quant(x, raw, dtype, in_dim, out_dim, threads=1)
        bound = O.gemv_bound(raw, dtype, in_dim, out_dim, x) + 1e-30
        covered = 0
        for r in range(world):
            row0, rows, y = results[r][ci]
            assert row0 == covered
            covered += rows
            assert np.all(np.abs(y.astype(np.float64) - full) <= bound)
        assert covered == out_dim


def test_plan_rules():
    from m3_avm_b200 import sharded

    assert sharded.shard_plan(12, 4096, 128256, 8, 7) == (112224, 16032, 16032, 112224 * 2304, 16032 * 2304)
    assert sharded.shard_plan(14, 4096, 10, 4, 3) == (9, 1, 3, 9 * 3360, 3360)
    assert sharded.shard_plan(14, 4096, 2, 4, 3) == (2, 0, 1, 2 * 3360, 0)
    assert sharded.shard_plan(12, 100, 256, 2, 0) is None   # rows would split blocks
    assert sharded.shard_plan(0, 4096, 16, 2, 0) is None    # no fused kernel
