"""The batch-1 Q4_K GEMV on tcgen05 kind::i8 (k_tc8_q4k) against the oracle.

Every row within 1e-5 * ||row||_1 * ||x||_inf of the oracle's port of the
reference matvec_q4k, over the shapes that exercise the kernel's row split:
fewer rows than SMs (one row per CTA), one tile per CTA with a partial last
CTA, several tiles per CTA, one and many super-blocks per row, and x with
large, tiny and zero super-blocks.  The kernel is off by default (tuning key
tc8 = 1 selects it); the same calls with tc8 = 0 take the mma.sync kernel, and
both must pass.
"""
import numpy as np
import pytest

from oracle import oracle as O
from m3_avm_b200 import synth

pytestmark = pytest.mark.gpu

SHAPES = [(256, 1), (256, 7), (4096, 100), (4096, 148), (4096, 1000), (4096, 14336), (2048, 18945),
          (8192, 28672), (14336, 4096), (4096, 37)]


@pytest.fixture(scope="module")
def m3():
    import torch

    from m3_avm_b200 import _lib
    from m3_avm_b200 import matvec_quant as MQ

    _lib.load()
    return torch, MQ


def _check(y, raw, in_dim, out_dim, x):
    ref = O.matvec_quant(x, raw, 12, in_dim, out_dim).astype(np.float64)
    bound = O.gemv_bound(raw, 12, in_dim, out_dim, x)
    err = np.abs(y.astype(np.float64) - ref)
    bad = np.nonzero(~(err <= bound))[0]
    assert bad.size == 0, f"rows {bad[:5]} err {err[bad[:5]]} bound {bound[bad[:5]]}"
    return float(np.max(err / bound))


@pytest.mark.parametrize("in_dim,out_dim", SHAPES, ids=[f"{o}x{i}" for i, o in SHAPES])
def test_tc8_matches_oracle(m3, in_dim, out_dim):
    torch, MQ = m3
    raw = synth.weights(12, in_dim, out_dim, seed=in_dim + out_dim)
    x = synth.activations(in_dim, seed=out_dim)
    if in_dim >= 2048:  # a super-block of huge values, one of tiny values, one of zeros
        x[256:512] *= np.float32(1e4)
        x[512:768] *= np.float32(1e-6)
        x[768:1024] = 0.0
    rd, xd = torch.from_numpy(raw).cuda(), torch.from_numpy(x).cuda()
    ys = {}
    for tc8 in (1, 0):
        MQ.set_tuning("tc8", tc8)
        try:
            y = MQ.matvec_quant_dev(xd, rd, 12, in_dim, out_dim)
            torch.cuda.synchronize()
            ys[tc8] = y.cpu().numpy()
        finally:
            MQ.set_tuning("tc8", 0)
        _check(ys[tc8], raw, in_dim, out_dim, x)
    assert MQ.device_status(0) == 0


def test_tc8_repeated_calls_are_deterministic(m3):
    """Same inputs, same bits: each row is summed in one fixed order."""
    torch, MQ = m3
    in_dim, out_dim = 4096, 14336
    raw = torch.from_numpy(synth.weights(12, in_dim, out_dim, seed=3)).cuda()
    x = torch.from_numpy(synth.activations(in_dim, seed=4)).cuda()
    MQ.set_tuning("tc8", 1)
    try:
        a = MQ.matvec_quant_dev(x, raw, 12, in_dim, out_dim)
        b = MQ.matvec_quant_dev(x, raw, 12, in_dim, out_dim)
        torch.cuda.synchronize()
    finally:
        MQ.set_tuning("tc8", 0)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
