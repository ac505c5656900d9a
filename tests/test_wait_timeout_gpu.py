"""A bounded device-side wait that runs out, on one GPU, without a fault.

The fused GEMV can gate its input on a device counter (the wait a sharded
decode step makes for the rows other GPUs store into it; the reference's
policy that failures never propagate is src/inference_gpu.rs:9-10).  Here the
counter never reaches its target: the kernel must give up after the
configured limit (10 ms instead of the 2 s default), report
kStatusPeerTimeout through the device status word, and leave the context
usable -- the next ordinary GEMV on the device still matches the oracle.
Nothing traps, faults or hangs: the wait is a poll with a wall-clock limit.
"""
import time

import numpy as np
import pytest

from oracle import oracle as O
from m3_avm_b200 import synth

pytestmark = pytest.mark.gpu

IN_DIM, OUT_DIM, DTYPE = 2048, 1024, 12
PEER_TIMEOUT = 8  # kStatusPeerTimeout


@pytest.fixture()
def cuda():
    import torch

    from m3_avm_b200 import _lib
    from m3_avm_b200 import matvec_quant as MQ

    _lib.load()
    torch.cuda.synchronize()
    MQ.device_status(0, clear=True)
    MQ.set_tuning("peer_wait_us", 10000)
    yield torch, MQ
    MQ.set_tuning("peer_wait_us", 2000000)
    torch.cuda.synchronize()
    MQ.device_status(0, clear=True)


def _inputs(torch):
    raw_h = synth.weights(DTYPE, IN_DIM, OUT_DIM, seed=31)
    x_h = synth.activations(IN_DIM, seed=32)
    return raw_h, x_h, torch.from_numpy(raw_h).cuda(), torch.from_numpy(x_h).cuda()


def test_gated_gemv_without_wait_equals_plain_gemv(cuda):
    torch, MQ = cuda
    raw_h, x_h, raw, x = _inputs(torch)
    ready = torch.full((1,), 5, dtype=torch.int32, device="cuda")
    y_gate = MQ.matvec_fused_wait_dev(x, raw, DTYPE, IN_DIM, OUT_DIM, ready=ready, target=5)
    y_fused = MQ.matvec_fused_dev(x, raw, DTYPE, IN_DIM, OUT_DIM)
    torch.cuda.synchronize()
    assert MQ.device_status(0) == 0
    assert np.array_equal(y_gate.cpu().numpy().view(np.uint32), y_fused.cpu().numpy().view(np.uint32))
    ref = O.matvec_quant(x_h, raw_h, DTYPE, IN_DIM, OUT_DIM)
    bound = O.gemv_bound(raw_h, DTYPE, IN_DIM, OUT_DIM, x_h)
    assert np.all(np.abs(y_gate.cpu().numpy().astype(np.float64) - ref) <= bound)


def test_wait_that_runs_out_reports_and_the_device_stays_usable(cuda):
    torch, MQ = cuda
    raw_h, x_h, raw, x = _inputs(torch)
    ready = torch.full((1,), 5, dtype=torch.int32, device="cuda")  # never reaches 6
    y = torch.empty(OUT_DIM, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    MQ.matvec_fused_wait_dev(x, raw, DTYPE, IN_DIM, OUT_DIM, ready=ready, target=6, y=y)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert waited < 1.0, waited  # the 10 ms limit, not the 2 s default
    status = MQ.device_status(0, clear=True)
    assert status & PEER_TIMEOUT, status
    assert MQ.device_status(0) == 0
    # an ordinary GEMV on the same device afterwards: still correct, no status
    y2 = MQ.matvec_quant_dev(x, raw, DTYPE, IN_DIM, OUT_DIM)
    torch.cuda.synchronize()
    ref = O.matvec_quant(x_h, raw_h, DTYPE, IN_DIM, OUT_DIM)
    bound = O.gemv_bound(raw_h, DTYPE, IN_DIM, OUT_DIM, x_h)
    assert np.all(np.abs(y2.cpu().numpy().astype(np.float64) - ref) <= bound)
    assert MQ.device_status(0) == 0


def test_peer_wait_limit_rejects_out_of_range(cuda):
    torch, MQ = cuda
    from m3_avm_b200 import _lib

    for bad in (0, -1, 60000001):
        with pytest.raises(_lib.M3GError):
            MQ.set_tuning("peer_wait_us", bad)
