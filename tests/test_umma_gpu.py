"""Batched Q4_K on the tcgen05 tensor cores (k_umma_q4k) against the oracle.

Every output row of every column within 1e-5 * ||row||_1 * ||x||_inf of the
oracle's fp32 result, at shapes that reach each part of the kernel:
* tiles cut between CTAs (one super-block per CTA; pieces finished by the
  CTA that completes the tile) and CTAs spanning several tiles;
* a ragged last tile (rows % 128 != 0), a single super-block per row;
* 8, 16, 32 and 64 accumulator columns, and more than 64 columns (two passes);
* columns of very different magnitudes and an all-zero column (the
  per-column power-of-two scaling of X);
* the batched-decode weight 28672 x 8192 at B = 16.
Also: the same call twice gives the same bits, and the path agrees with the
8-column kernel and with per-column GEMVs.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def m3():
    import m3_avm_b200 as pkg
    from m3_avm_b200 import _lib

    _lib.load()
    return pkg


def _bound(raw, in_dim, out_dim, x):
    return O.gemv_bound(raw, 12, in_dim, out_dim, x) + 1e-30


def _run(m3, X, raw, in_dim, out_dim):
    import torch

    xd = torch.from_numpy(np.ascontiguousarray(X)).cuda()
    rd = torch.from_numpy(raw).cuda()
    Y = m3.matvec_quant.matvec_quant_dev(xd, rd, 12, in_dim, out_dim)
    torch.cuda.synchronize()
    return Y.cpu().numpy()


def _check(Y, raw, in_dim, out_dim, X, cols=None):
    worst = 0.0
    for b in (range(X.shape[0]) if cols is None else cols):
        ref = O.matvec_quant(X[b], raw, 12, in_dim, out_dim)
        err = np.abs(Y[b].astype(np.float64) - ref.astype(np.float64))
        bound = _bound(raw, in_dim, out_dim, X[b])
        bad = np.nonzero(err > bound)[0]
        assert bad.size == 0, f"column {b} rows {bad[:5]} err {err[bad[:5]]} bound {bound[bad[:5]]}"
        worst = max(worst, float(np.max(err / bound)))
    return worst


@pytest.mark.parametrize("in_dim,out_dim,batch", [
    (768, 37, 2),        # one tile, three one-super-block pieces
    (2304, 1000, 8),     # 8 tiles x 9 super-blocks, one super-block per CTA
    (2304, 1000, 9),
    (4096, 513, 16),     # ragged last tile (1 row)
    (256, 16, 7),        # one super-block, one CTA, a whole tile
    (8192, 2048, 17),    # 32 accumulator columns; CTAs span tiles
    (8192, 2048, 33),    # 64 accumulator columns
    (4096, 4096, 64),
    (1024, 300, 70),     # two passes: 64 + 6 columns
])
def test_umma_batched_q4k_matches_oracle(m3, in_dim, out_dim, batch):
    raw = m3.synth.weights(12, in_dim, out_dim, seed=in_dim + 7 * batch)
    X = m3.synth.activations(in_dim, seed=90 + batch, batch=batch)
    Y = _run(m3, X, raw, in_dim, out_dim)
    assert _check(Y, raw, in_dim, out_dim, X) < 0.5
    assert m3.matvec_quant.device_status(0) == 0


def test_umma_column_scaling(m3):
    """Columns 1e-6, 1, 1e4 in magnitude and an all-zero column."""
    in_dim, out_dim = 4096, 700
    raw = m3.synth.weights(12, in_dim, out_dim, seed=11)
    X = m3.synth.activations(in_dim, seed=12, batch=5)
    X[0] *= np.float32(1e-6)
    X[2] *= np.float32(1e4)
    X[3] = 0.0
    X[4, ::7] *= np.float32(300.0)  # a few large entries in one column
    Y = _run(m3, X, raw, in_dim, out_dim)
    _check(Y, raw, in_dim, out_dim, X)
    assert np.all(Y[3] == 0.0)


@pytest.mark.parametrize("peak", [3.999, 4.0, 1.0001, 65504.0])
def test_umma_scaled_magnitude_near_fp16_limits(m3, peak):
    """Largest |x| just below / at a power of two: scaled values near 2^15 and
    group sums of 32 of them (a constant column sums to 32x its maximum)."""
    in_dim, out_dim = 2048, 300
    raw = m3.synth.weights(12, in_dim, out_dim, seed=21)
    X = m3.synth.activations(in_dim, seed=22, batch=4)
    X = (X / np.abs(X).max(axis=1, keepdims=True) * np.float32(peak)).astype(np.float32)
    X[1] = np.float32(peak)
    X[2, ::2] = np.float32(-peak)
    Y = _run(m3, X, raw, in_dim, out_dim)
    assert np.all(np.isfinite(Y))
    _check(Y, raw, in_dim, out_dim, X)


def test_umma_batched_decode_weight(m3):
    in_dim, out_dim, batch = 8192, 28672, 16
    raw = m3.synth.weights(12, in_dim, out_dim, seed=4242)
    X = m3.synth.activations(in_dim, seed=4243, batch=batch)
    Y = _run(m3, X, raw, in_dim, out_dim)
    assert _check(Y, raw, in_dim, out_dim, X, cols=[0, 5, 15]) < 0.5


def test_umma_repeatable_bits(m3):
    """Tiles finished from several CTAs' pieces add them in CTA order."""
    in_dim, out_dim, batch = 8192, 3000, 24
    raw = m3.synth.weights(12, in_dim, out_dim, seed=5)
    X = m3.synth.activations(in_dim, seed=6, batch=batch)
    a = _run(m3, X, raw, in_dim, out_dim)
    b = _run(m3, X, raw, in_dim, out_dim)
    assert np.all(np.isfinite(a))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_umma_agrees_with_gemm8_and_per_column(m3):
    in_dim, out_dim, batch = 4096, 4096, 12
    raw = m3.synth.weights(12, in_dim, out_dim, seed=3)
    X = m3.synth.activations(in_dim, seed=4, batch=batch)
    a = _run(m3, X, raw, in_dim, out_dim)
    mq = m3.matvec_quant
    mq.set_tuning("umma", 0)
    try:
        b = _run(m3, X, raw, in_dim, out_dim)
        mq.set_tuning("gemm8", 0)
        c = _run(m3, X, raw, in_dim, out_dim)
    finally:
        mq.set_tuning("umma", 1)
        mq.set_tuning("gemm8", 1)
    for k in range(batch):
        bound = _bound(raw, in_dim, out_dim, X[k])
        assert np.all(np.abs(a[k].astype(np.float64) - b[k]) <= 2 * bound)
        assert np.all(np.abs(a[k].astype(np.float64) - c[k]) <= 2 * bound)
