"""m3g_matvec_greedy_noalloc: the greedy vocab head that allocates no device
memory, checked on two calls in a row against the existing entry points (the
GEMV of m3g_matvec_quant_dev, then the first index of the maximum) and
against the oracle's logits (the pick must be a row whose oracle logit is
within the GEMV tolerance of the largest).  Collected last so it also runs
after every other GPU test."""
import numpy as np
import pytest

from oracle import oracle as O
from m3_avm_b200 import synth

pytestmark = pytest.mark.gpu

IN_DIM, OUT_DIM, DTYPE = 2048, 50000, 14


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    from m3_avm_b200 import _lib

    _lib.load()
    return torch


def expected_pick(torch, MQ, x, raw, bound):
    """Greedy pick of the existing GEMV's logits, plus the set of rows within
    the GEMV tolerance of the maximum (any of them is an acceptable pick)."""
    y = MQ.matvec_quant_dev(x, raw, DTYPE, IN_DIM, OUT_DIM)
    torch.cuda.synchronize()
    yh = y.cpu().numpy().astype(np.float64)
    top = yh.max()
    near = set(np.nonzero(yh >= top - 2 * bound)[0].tolist())
    return int(np.argmax(yh)), near


def test_noalloc_greedy_matches_existing_entry_twice(torch_cuda):
    torch = torch_cuda
    from m3_avm_b200 import matvec_quant as MQ

    dev = torch.device("cuda:0")
    raw_h = synth.weights(DTYPE, IN_DIM, OUT_DIM, seed=5)
    raw = torch.from_numpy(raw_h).to(dev)
    xs = [synth.activations(IN_DIM, seed=s) for s in (6, 7)]
    token = torch.full((1,), -7, dtype=torch.int32, device=dev)
    # first call: sets up the scratch address for this device
    MQ.matvec_greedy_noalloc(torch.from_numpy(xs[0]).to(dev), raw, DTYPE, IN_DIM, OUT_DIM, token=token)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    for xh in xs:  # two calls in a row, each checked
        x = torch.from_numpy(xh).to(dev)
        bound = float(np.max(O.gemv_bound(raw_h, DTYPE, IN_DIM, OUT_DIM, xh)))
        want, near = expected_pick(torch, MQ, x, raw, bound)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        MQ.matvec_greedy_noalloc(x, raw, DTYPE, IN_DIM, OUT_DIM, token=token)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info(dev)[0] == free_before  # nothing allocated by the call
        got = int(token.item())
        assert got == want or got in near, (got, want, sorted(near)[:5])
        # the oracle's logits: the pick is the top row, or a row that the
        # per-row tolerance cannot tell apart from it
        ref = O.matvec_quant(xh, raw_h, DTYPE, IN_DIM, OUT_DIM).astype(np.float64)
        rb = O.gemv_bound(raw_h, DTYPE, IN_DIM, OUT_DIM, xh)
        assert ref[got] + rb[got] >= np.max(ref - rb), (got, int(np.argmax(ref)))
    assert torch.cuda.mem_get_info(dev)[0] <= free0 + 0  # no growth after setup either


def test_noalloc_greedy_rejects_rows_beyond_scratch(torch_cuda):
    torch = torch_cuda
    from m3_avm_b200 import _lib
    from m3_avm_b200 import matvec_quant as MQ

    dev = torch.device("cuda:0")
    x = torch.zeros(IN_DIM, device=dev)
    raw = torch.zeros(16, dtype=torch.uint8, device=dev)
    with pytest.raises(_lib.M3GError, match="no-alloc scratch"):
        MQ.matvec_greedy_noalloc(x, raw, DTYPE, IN_DIM, 262145)
