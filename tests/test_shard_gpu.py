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


def _captured_first_call(q):
    """Child process: the very first GEMV of the process is a sharded matvec
    captured into a CUDA graph (nothing may allocate inside the capture)."""
    import torch

    from m3_avm_b200 import sharded, synth

    try:
        in_dim, out_dim, dtype = 4096, 2048, 12
        raw = synth.weights(dtype, in_dim, out_dim, seed=21)
        x = synth.activations(in_dim, seed=22)
        s = sharded.ShardedOffload(0, 0, 1, sharded.unique_id(), in_dim, out_dim, timeout_s=60)
        assert s.upload(0, dtype, raw, in_dim, out_dim)
        xd = torch.from_numpy(x).cuda()
        yd = torch.zeros(s.gather_len(0), device="cuda")
        st = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st, capture_error_mode="thread_local"):
            s.matvec_dev(0, xd, yd, stream=st.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        y = yd[:out_dim].cpu().numpy()
        del g
        s.close()
        q.put(("ok", y.tobytes()))
    except Exception as e:  # reported to the parent
        q.put(("error", repr(e)))


def test_world1_matvec_captured_as_first_call():
    import multiprocessing as mp

    from m3_avm_b200 import synth

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_captured_first_call, args=(q,))
    p.start()
    kind, payload = q.get(timeout=300)
    p.join(60)
    assert kind == "ok", payload
    y = np.frombuffer(payload, np.float32)
    in_dim, out_dim, dtype = 4096, 2048, 12
    _check(y, synth.weights(dtype, in_dim, out_dim, seed=21), dtype, in_dim, out_dim, synth.activations(in_dim, seed=22))


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


def _rank(rank, world, uid, p2p, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    torch.cuda.set_device(rank)
    from m3_avm_b200 import matvec_quant as MQ
    from m3_avm_b200 import sharded, synth

    try:
        MQ.set_tuning("shard_p2p", p2p)
        s = sharded.ShardedOffload(rank, rank, world, uid, 4096, 128256, timeout_s=60)
        out = []
        for tidx, (dtype, in_dim, out_dim) in enumerate(SHAPES2):
            raw = synth.weights(dtype, in_dim, out_dim, seed=11 + tidx)
            assert s.upload(tidx, dtype, raw, in_dim, out_dim)
            for call in range(3):  # consecutive calls alternate the exchange halves
                x = synth.activations(in_dim, seed=12 + call)
                out.append(s.matvec(tidx, x, in_dim, out_dim).tobytes())
            X = synth.activations(in_dim, seed=20, batch=3)  # batch > 1: the NCCL all-gather
            out.append(s.matvec(tidx, X, in_dim, out_dim).tobytes())
            # device form inside a captured CUDA graph, replayed twice
            xd = torch.from_numpy(synth.activations(in_dim, seed=12)).cuda()
            yd = torch.zeros(s.gather_len(tidx), device="cuda")
            st = torch.cuda.Stream()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st, capture_error_mode="thread_local"):
                s.matvec_dev(tidx, xd, yd, stream=st.cuda_stream)
            for _ in range(2):
                g.replay()
                torch.cuda.synchronize()
                out.append(yd[:out_dim].cpu().numpy().tobytes())
            del g
        exchange = s.exchange
        status = MQ.device_status(rank)
        s.close()
        q.put((rank, (exchange, status, out)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))


SHAPES2 = [(14, 4096, 128256), (12, 4096, 14337), (12, 4096, 3)]


@pytest.mark.parametrize("p2p,exchange", [(1, "peer-stores"), (0, "nccl")], ids=["peer-stores", "nccl"])
def test_world2_all_ranks_hold_full_output(p2p, exchange):
    """Both ranks hold the whole output after every call, equal to the oracle,
    with the rows exchanged by peer stores from the GEMV epilogue and by the
    NCCL all-gather; three calls in a row (the peer form alternates its
    exchange halves), a batched call, and graph replays.  A 3-row tensor
    leaves rank 1 without rows: it takes the NCCL path in both modes."""
    import multiprocessing as mp

    import torch

    from m3_avm_b200 import sharded, synth

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    uid = sharded.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, p2p, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert res[r][0] == exchange and res[r][1] == 0
    k = 0
    for tidx, (dtype, in_dim, out_dim) in enumerate(SHAPES2):
        raw = synth.weights(dtype, in_dim, out_dim, seed=11 + tidx)
        for call in range(3):
            x = synth.activations(in_dim, seed=12 + call)
            ys = [np.frombuffer(res[r][2][k], np.float32) for r in range(world)]
            assert np.array_equal(ys[0], ys[1])
            _check(ys[0], raw, dtype, in_dim, out_dim, x)
            if call == 0:
                first = ys[0]
            k += 1
        X = synth.activations(in_dim, seed=20, batch=3)
        Ys = [np.frombuffer(res[r][2][k], np.float32).reshape(3, out_dim) for r in range(world)]
        assert np.array_equal(Ys[0], Ys[1])
        for b in range(3):
            _check(Ys[0][b], raw, dtype, in_dim, out_dim, X[b])
        k += 1
        for _ in range(2):  # graph replays of the first call's input give its bits
            for r in range(world):
                assert np.array_equal(np.frombuffer(res[r][2][k], np.float32), first)
            k += 1
