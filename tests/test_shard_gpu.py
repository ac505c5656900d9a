"""Row-sharded GEMV with the NCCL all-gather, on the GPU.

* world 1 on one GPU: the communicator, the in-place all-gather and the
  output layout, against the oracle;
* a rank that never joins: create() gives up with M3G_ETIMEOUT (host-side
  failure detection; nothing waits on the GPU);
* world 2 on two GPUs when present: every rank holds the full output.
"""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _check(y, raw, dtype, in_dim, out_dim, x):
    ref = O.matvec_quant(x, raw, dtype, in_dim, out_dim)
    bound = O.gemv_bound(raw, dtype, in_dim, out_dim, x) + 1e-30
    assert np.all(np.abs(y.astype(np.float64) - ref) <= bound)


def test_world1_matches_oracle():
    import torch

    from m3_avm_b200 import sharded, synth

    s = sharded.ShardedOffload(0, 0, 1, sharded.unique_id(), 4096, 128256, timeout_s=60)
    try:
        for tidx, (dtype, in_dim, out_dim) in enumerate([(14, 4096, 8192), (12, 4096, 1000), (8, 2048, 96)]):
            raw = synth.weights(dtype, in_dim, out_dim, seed=5 + tidx)
            x = synth.activations(in_dim, seed=6)
            assert s.upload(tidx, dtype, raw, in_dim, out_dim)
            _check(s.matvec(tidx, x, in_dim, out_dim), raw, dtype, in_dim, out_dim, x)
            X = synth.activations(in_dim, seed=7, batch=3)
            Y = s.matvec(tidx, X, in_dim, out_dim)
            for b in range(3):
                _check(Y[b], raw, dtype, in_dim, out_dim, X[b])
            # device form, batch 1: y[0:out] is the output
            xd = torch.from_numpy(x).cuda()
            yd = torch.zeros(s.gather_len(tidx), device="cuda")
            s.matvec_dev(tidx, xd, yd)
            torch.cuda.synchronize()
            _check(yd[:out_dim].cpu().numpy(), raw, dtype, in_dim, out_dim, x)
        assert not s.upload(9, 12, synth.weights(12, 100 * 256 // 100, 100, 1)[:-1], 256, 100)
    finally:
        s.close()


def _lonely_rank(uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from m3_avm_b200 import _lib, sharded

    try:
        sharded.ShardedOffload(0, 0, 2, uid, 16, 16, timeout_s=3.0)
        q.put(("joined", 0))
    except _lib.M3GError as e:
        q.put(("error", e.code))


def test_rank_that_never_joins_times_out():
    import multiprocessing as mp

    from m3_avm_b200 import _lib, sharded

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(sharded.unique_id(), q))
    p.start()
    p.join(120)
    assert p.exitcode == 0
    assert q.get(timeout=5) == ("error", _lib.M3G_ETIMEOUT)


def _rank(rank, world, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    torch.cuda.set_device(rank)
    from m3_avm_b200 import sharded, synth

    s = sharded.ShardedOffload(rank, rank, world, uid, 4096, 128256, timeout_s=60)
    out = []
    for tidx, (dtype, in_dim, out_dim) in enumerate([(14, 4096, 128256), (12, 4096, 14337)]):
        raw = synth.weights(dtype, in_dim, out_dim, seed=11 + tidx)
        x = synth.activations(in_dim, seed=12)
        assert s.upload(tidx, dtype, raw, in_dim, out_dim)
        out.append(s.matvec(tidx, x, in_dim, out_dim))
    s.close()
    q.put((rank, [o.tobytes() for o in out]))


def test_world2_all_ranks_hold_full_output():
    import multiprocessing as mp

    import torch

    from m3_avm_b200 import sharded, synth

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    uid = sharded.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for tidx, (dtype, in_dim, out_dim) in enumerate([(14, 4096, 128256), (12, 4096, 14337)]):
        raw = synth.weights(dtype, in_dim, out_dim, seed=11 + tidx)
        x = synth.activations(in_dim, seed=12)
        ys = [np.frombuffer(res[r][tidx], np.float32) for r in range(world)]
        assert np.array_equal(ys[0], ys[1])
        _check(ys[0], raw, dtype, in_dim, out_dim, x)
