"""GPU parity: the sm_100a kernels through the C ABI against the CPU oracle.

* decoders: bit-exact f32 output for every dtype, random and known-answer blocks;
* GEMV: every output row within 1e-5 * ||row||_1 * ||x||_inf of the oracle's
  reference-order fp32 result (the bound the port is held to), at small odd
  shapes (blocks straddling rows), the benchmark shapes, and through the
  streaming and the generic kernels alike;
* the reference's own known answers through the GPU path;
* the GpuOffload-shaped API and its failure rules.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests import refcases as R

pytestmark = pytest.mark.gpu

BLOCK = {2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 144), 14: (256, 210)}


@pytest.fixture(scope="module")
def m3():
    import m3_avm_b200 as pkg
    from m3_avm_b200 import _lib

    _lib.load()
    return pkg


def gemv_bound(raw, dtype, in_dim, out_dim, x):
    return O.gemv_bound(raw, dtype, in_dim, out_dim, x) + 1e-30


def check_gemv(y, raw, dtype, in_dim, out_dim, x, ref=None):
    if ref is None:
        ref = O.matvec_quant(x, raw, dtype, in_dim, out_dim)
    assert ref is not None and y is not None
    assert y.shape == (out_dim,)
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    bound = gemv_bound(raw, dtype, in_dim, out_dim, x)
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, f"rows {bad[:5]} err {err[bad[:5]]} bound {bound[bad[:5]]}"
    return float(np.max(err / bound))


# ---------------------------------------------------------------- decoders, bit-exact
def _bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | both_nan))


@pytest.mark.parametrize("dtype", [2, 8, 12, 13, 14])
@pytest.mark.parametrize("nblocks", [1, 7, 4096])
def test_dequant_bit_exact_random(m3, dtype, nblocks):
    be, _ = BLOCK[dtype]
    raw = m3.synth.weights(dtype, be, nblocks, seed=99 + nblocks + dtype)
    n = be * nblocks
    dst = np.zeros(n, np.float32)
    assert m3.quant.dequantize(raw, dtype, dst, n)
    assert _bits_equal(dst, O.dequantize(raw, dtype, n))


@pytest.mark.parametrize("dtype", [2, 8, 12, 14])
def test_dequant_bit_exact_special_scales(m3, dtype):
    """Scale fields that are f16 subnormal, zero, negative zero, max, inf and NaN."""
    be, bb = BLOCK[dtype]
    specials = [0x0001, 0x03FF, 0x0000, 0x8000, 0x7BFF, 0xFBFF, 0x7C00, 0x7E00, 0x3C00, 0xBC00]
    raw = m3.synth.weights(dtype, be, len(specials) ** 2, seed=5).reshape(-1, bb).copy()
    dpos = {2: [0], 8: [0], 12: [0, 2], 14: [208]}[dtype]
    k = 0
    for a in specials:
        for b in specials:
            vals = [a, b]
            for i, p in enumerate(dpos):
                raw[k, p] = vals[i] & 0xFF
                raw[k, p + 1] = vals[i] >> 8
            k += 1
    raw = raw.reshape(-1)
    n = be * len(specials) ** 2
    dst = np.zeros(n, np.float32)
    assert m3.quant.dequantize(raw, dtype, dst, n)
    assert _bits_equal(dst, O.dequantize(raw, dtype, n))


def test_dequant_f32_f16(m3):
    src = np.array([1.0, -2.5, 3e-39, np.inf], np.float32).view(np.uint8)
    dst = np.zeros(4, np.float32)
    assert m3.quant.dequantize(src, 0, dst, 4)
    assert _bits_equal(dst, O.dequantize(src, 0, 4))
    h = np.arange(0, 65536, 7, dtype=np.uint16)
    dst = np.zeros(h.size, np.float32)
    assert m3.quant.dequantize(h.view(np.uint8), 1, dst, h.size)
    assert _bits_equal(dst, h.view(np.float16).astype(np.float32))


def test_dequant_reference_kats(m3):
    """src/quant.rs:288-370 through the GPU decoders."""
    src = bytearray(18)
    src[1] = 0x3C
    src[2:] = b"\x88" * 16
    dst = np.full(32, 99.0, np.float32)
    m3.quant.dequant_q4_0(src, dst, 32)
    assert np.all(np.abs(dst) < 1e-5)
    src = bytearray(144)
    src[1] = 0x3C
    src[16:] = b"\x88" * 128
    src[4:16] = b"\x10" * 12
    dst = np.zeros(256, np.float32)
    m3.quant.dequant_q4_k(src, dst, 256)
    assert dst[0] == 128.0 and np.all(dst[:128] == 128.0) and np.all(dst[128:] == 0.0)
    src = bytearray(210)
    src[209] = 0x3C
    src[192:208] = b"\xff" * 16
    dst = np.zeros(256, np.float32)
    m3.quant.dequant_q6_k(src, dst, 256)
    assert np.all(dst == 32.0)


def test_dequant_failure_rules(m3):
    dst = np.zeros(512, np.float32)
    raw = R.synth_q4k(512)
    assert not m3.quant.dequantize(raw, 12, dst, 100)
    assert not m3.quant.dequantize(bytes(10), 14, dst, 256)
    assert not m3.quant.dequantize(bytes(10), 8, dst, 32)
    assert not m3.quant.dequantize(bytes(10), 3, dst, 32)
    with pytest.raises(AssertionError):
        m3.quant.dequantize(bytes(10), 12, dst, 256)
    with pytest.raises(AssertionError):
        m3.quant.dequant_q4_k(raw, dst, 100)


# ---------------------------------------------------------------- GEMV vs oracle
SHAPES = [
    # (in_dim, out_dim): straddling blocks, tiny, ragged unit counts, config rows
    (16, 16), (32, 16), (48, 32), (256, 16), (512, 300), (1536, 96), (2048, 520), (4096, 64), (8192, 48),
    (14336, 24), (4096, 4096),
]


KERNELS = {
    # tuning that selects each kernel where the shape allows it
    "mma": {},
    "mma_2tile_kc8": {"mma_tps": 2, "mma_kc": 8},
    "mma_2cta": {"mma_ctas": 2},
    "mma_wk16": {"mma_wk": 16},
    "mma_wk8": {"mma_wk": 8},
    "mma_rowcopy": {"mma_cg": 1},
    "mma_coresident": {"mma_coresident": 1, "mma_pre": 0},
    "stream": {"mma": 0},
    "generic": {"force_generic": 1},
}
DEFAULT_TUNING = {"mma": 1, "force_generic": 0, "mma_tps": 0, "mma_kc": 16, "mma_ctas": 1, "mma_wk": 0, "mma_cg": 4, "mma_coresident": 0, "mma_pre": 1}


@pytest.fixture(params=list(KERNELS))
def kernel(request, m3):
    for k, v in KERNELS[request.param].items():
        m3.matvec_quant.set_tuning(k, v)
    yield request.param
    for k, v in DEFAULT_TUNING.items():
        m3.matvec_quant.set_tuning(k, v)


@pytest.mark.parametrize("dtype", [2, 8, 12, 14])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemv_matches_oracle(m3, kernel, dtype, shape):
    in_dim, out_dim = shape
    be, _ = BLOCK[dtype]
    if (in_dim * out_dim) % be:
        pytest.skip("not a whole number of blocks")
    raw = m3.synth.weights(dtype, in_dim, out_dim, seed=in_dim * 7 + out_dim + dtype)
    x = m3.synth.activations(in_dim, seed=in_dim + 3)
    y = m3.matvec_quant.matvec_quant(x, raw, dtype, in_dim, out_dim)
    check_gemv(y, raw, dtype, in_dim, out_dim, x)


@pytest.mark.parametrize("dtype", [2, 8, 12, 14])
def test_generic_kernel_matches_oracle(m3, dtype):
    """The row-straddling fallback kernel on shapes the streaming kernel also serves."""
    in_dim, out_dim = 4096, 40
    raw = m3.synth.weights(dtype, in_dim, out_dim, seed=17)
    x = m3.synth.activations(in_dim, seed=18)
    m3.matvec_quant.set_tuning("force_generic", 1)
    try:
        y = m3.matvec_quant.matvec_quant(x, raw, dtype, in_dim, out_dim)
    finally:
        m3.matvec_quant.set_tuning("force_generic", 0)
    check_gemv(y, raw, dtype, in_dim, out_dim, x)


def test_reference_kats_on_gpu(m3):
    """src/matvec_quant.rs:411-581 known answers and parity cases, through the GPU."""
    M = m3.matvec_quant
    x = R.x_ones_half(16)
    y = M.matvec_q4k(x, R.raw_q4k_ones(256), 16, 16)
    assert np.all(np.abs(y - x.sum()) < 1e-3)
    raw = R.q4k_pattern_37_11(32, 16)
    x = R.x_sin(32, 0.13, 0.7)
    y = M.matvec_q4k(x, raw, 32, 16)
    y_ref = O.matvec_dense(x, O.dequantize(raw, 12, 512), 32, 16)
    assert np.max(np.abs(y - y_ref)) < 1e-2
    raw = R.q4k_pattern_53_29(256, 16, dmin_hi=0xBC)
    x = R.x_sin(256, 0.31, 1.7)
    a = O.matvec_q4k_avx2(x, raw, 256, 16)
    b = M.matvec_q4k(x, raw, 256, 16)
    assert np.max(np.abs(a - b)) / np.max(np.abs(a)) < 1e-4
    check_gemv(b, raw, 12, 256, 16, x, ref=a)
    raw = R.q4k_pattern_53_29(48, 32)
    x = R.x_sin(48, 0.11, 0.9)
    check_gemv(M.matvec_q4k(x, raw, 48, 32), raw, 12, 48, 32, x)
    raw = R.q8_0_pattern(64)
    x = R.x_q8(8)
    y = M.matvec_q8_0(x, raw, 8, 8)
    assert np.max(np.abs(y - O.matvec_dense(x, O.dequantize(raw, 8, 64), 8, 8))) < 1e-4
    for n_in, n_out in ((1536, 64), (256, 96)):
        raw = R.synth_q4k(n_in * n_out)
        x = R.x_sin(n_in, 0.017, 0.6)
        check_gemv(M.matvec_q4k(x, raw, n_in, n_out), raw, 12, n_in, n_out, x)
        raw = R.synth_q6k(n_in * n_out)
        check_gemv(M.matvec_q6k(x, raw, n_in, n_out), raw, 14, n_in, n_out, x)


def test_dispatcher_none_rules_on_gpu(m3):
    """src/matvec_quant.rs:533-553."""
    M = m3.matvec_quant
    x8 = np.ones(8, np.float32)
    assert M.matvec_quant(x8, bytes(64), 0, 8, 2) is None
    assert M.matvec_quant(x8, bytes(10), 12, 32, 8) is None
    assert M.matvec_quant(x8, bytes(144), 12, 7, 5) is None
    raw = R.raw_q4k_ones(256)
    assert M.matvec_quant(np.ones(4, np.float32), raw, 12, 16, 16) is None
    x16 = np.full(16, 0.5, np.float32)
    a = M.matvec_quant(x16, raw, 12, 16, 16)
    b = M.matvec_q4k(x16, raw, 16, 16)
    assert np.all(np.abs(a - b) < 1e-6)
    # dtype 13 runs the Q4_K kernel, a longer raw is accepted and truncated
    c = M.matvec_quant(x16, np.concatenate([raw, np.zeros(50, np.uint8)]), 13, 16, 16)
    assert np.array_equal(a, c)


def test_gemv_linearity(m3):
    """A size-independent property: W(a x1 + x2) == a W x1 + W x2 within the bound."""
    import torch

    in_dim, out_dim = 4096, 14336
    raw = m3.synth.weights(12, in_dim, out_dim, seed=77)
    x1 = m3.synth.activations(in_dim, seed=1)
    x2 = m3.synth.activations(in_dim, seed=2)
    xs = np.stack([x1, x2, (np.float32(0.5) * x1 + x2).astype(np.float32)])
    d_raw = torch.from_numpy(raw).cuda()
    Y = m3.matvec_quant.matvec_quant_dev(torch.from_numpy(xs).cuda(), d_raw, 12, in_dim, out_dim).cpu().numpy()
    bound = 3 * gemv_bound(raw, 12, in_dim, out_dim, xs[2])
    assert np.all(np.abs(Y[2] - (0.5 * Y[0] + Y[1])) <= bound)


def test_gemv_batched_dev_matches_oracle(m3):
    import torch

    in_dim, out_dim, batch = 2048, 1000, 5
    raw = m3.synth.weights(14, in_dim, out_dim, seed=31)
    X = m3.synth.activations(in_dim, seed=32, batch=batch)
    Y = m3.matvec_quant.matvec_quant_dev(torch.from_numpy(X).cuda(), torch.from_numpy(raw).cuda(), 14, in_dim,
                                         out_dim).cpu().numpy()
    for b in range(batch):
        check_gemv(Y[b], raw, 14, in_dim, out_dim, X[b])


# ---------------------------------------------------------------- benchmark shapes
@pytest.mark.parametrize("dtype,in_dim,out_dim", [
    (12, 4096, 4096),     # single Q4_K GEMV
    (12, 4096, 14336),    # FFN gate/up
    (14, 14336, 4096),    # FFN down
    (8, 4096, 4096),      # Q8_0
    (2, 4096, 4096),      # Q4_0
    (14, 4096, 128256),   # vocab head
    (12, 8192, 28672),    # batched-decode weight, one column
])
def test_benchmark_shapes_match_oracle(m3, dtype, in_dim, out_dim):
    import torch

    raw = m3.synth.weights(dtype, in_dim, out_dim, seed=2024 + dtype)
    x = m3.synth.activations(in_dim, seed=7)
    y = m3.matvec_quant.matvec_quant_dev(torch.from_numpy(x).cuda(), torch.from_numpy(raw).cuda(), dtype, in_dim,
                                         out_dim).cpu().numpy()
    worst = check_gemv(y, raw, dtype, in_dim, out_dim, x)
    assert worst < 0.5


# ---------------------------------------------------------------- offload API
def test_offload_api_rules(m3):
    G = m3.inference_gpu.GpuOffload
    g = G.try_new(4096, 14336)
    assert g is not None
    raw = m3.synth.weights(12, 4096, 512, seed=3)
    assert g.upload(5, 12, raw, 4096, 512)
    assert g.offloaded(5) and not g.offloaded(6) and g.tensor_count() == 1
    assert not g.upload(6, 0, raw, 4096, 512)                 # no fused kernel for F32
    assert not g.upload(6, 12, raw[:-1], 4096, 512)           # raw_len != quant_raw_len
    assert not g.upload(6, 12, raw, 0, 512)
    x = m3.synth.activations(4096, seed=4)
    y = g.matvec(5, x, 4096, 512)
    check_gemv(y, raw, 12, 4096, 512, x)
    assert g.calls == 1
    assert g.matvec(5, x, 4096, 511) is None                  # dims differ from upload
    assert g.matvec(9, x, 4096, 512) is None                  # not resident
    raw6 = m3.synth.weights(14, 2048, 300, seed=8)
    assert g.upload(7, 14, raw6, 2048, 300)
    X = m3.synth.activations(2048, seed=9, batch=3)
    Y = g.matvec_batch(7, X, 2048, 300)
    for b in range(3):
        check_gemv(Y[b], raw6, 14, 2048, 300, X[b])
    # re-upload replaces
    raw2 = m3.synth.weights(12, 4096, 512, seed=10)
    assert g.upload(5, 12, raw2, 4096, 512)
    check_gemv(g.matvec(5, x, 4096, 512), raw2, 12, 4096, 512, x)
    g.close()


def test_status_word_clean_after_suite(m3):
    assert m3.matvec_quant.device_status(0) == 0


# ---------------------------------------------------------------- batched Q4_K (8 columns per pass)
@pytest.mark.parametrize("in_dim,out_dim,batch", [(768, 37, 2), (2304, 1000, 8), (2304, 1000, 9), (4096, 513, 16),
                                                  (8192, 2048, 33), (256, 16, 7)])
def test_gemm8_batched_q4k_matches_oracle(m3, in_dim, out_dim, batch):
    import torch

    raw = m3.synth.weights(12, in_dim, out_dim, seed=in_dim + batch)
    X = m3.synth.activations(in_dim, seed=40 + batch, batch=batch) * np.float32(2.0)
    dev = torch.device("cuda:0")
    xd = torch.from_numpy(X).to(dev)
    rd = torch.from_numpy(raw).to(dev)
    m3.matvec_quant.set_tuning("umma", 0)  # the 8-column mma.sync kernel
    try:
        Y = m3.matvec_quant.matvec_quant_dev(xd, rd, 12, in_dim, out_dim)
        torch.cuda.synchronize()
    finally:
        m3.matvec_quant.set_tuning("umma", 1)
    Yh = Y.cpu().numpy()
    for b in range(batch):
        check_gemv(Yh[b], raw, 12, in_dim, out_dim, X[b])


def test_gemm8_equals_per_column_gemv(m3):
    """The batched kernel and B single GEMVs agree within the bound (both are
    checked against the oracle above); the switch routes through either."""
    import torch

    in_dim, out_dim, batch = 4096, 4096, 12
    raw = m3.synth.weights(12, in_dim, out_dim, seed=3)
    X = m3.synth.activations(in_dim, seed=4, batch=batch)
    dev = torch.device("cuda:0")
    xd, rd = torch.from_numpy(X).to(dev), torch.from_numpy(raw).to(dev)
    m3.matvec_quant.set_tuning("umma", 0)  # the 8-column mma.sync kernel
    try:
        a = m3.matvec_quant.matvec_quant_dev(xd, rd, 12, in_dim, out_dim)
        m3.matvec_quant.set_tuning("gemm8", 0)
        b = m3.matvec_quant.matvec_quant_dev(xd, rd, 12, in_dim, out_dim)
    finally:
        m3.matvec_quant.set_tuning("gemm8", 1)
        m3.matvec_quant.set_tuning("umma", 1)
    torch.cuda.synchronize()
    for k in range(batch):
        bound = gemv_bound(raw, 12, in_dim, out_dim, X[k])
        assert np.all(np.abs(a[k].cpu().numpy().astype(np.float64) - b[k].cpu().numpy()) <= 2 * bound)


def test_offload_replayed_calls_follow_reuploads_and_batch_sizes(m3):
    """Host-buffer offload calls replay a captured graph per tensor: a new
    upload of the same index, a different batch and a larger staging buffer
    must each give the oracle's result for the current weights."""
    g = m3.inference_gpu.GpuOffload.try_new(4096, 1024)
    assert g is not None
    raw_a = m3.synth.weights(12, 4096, 1024, seed=61)
    raw_b = m3.synth.weights(12, 4096, 1024, seed=62)
    x = m3.synth.activations(4096, seed=63)
    assert g.upload(3, 12, raw_a, 4096, 1024)
    for _ in range(2):  # the second call replays the graph
        check_gemv(g.matvec(3, x, 4096, 1024), raw_a, 12, 4096, 1024, x)
    assert g.upload(3, 12, raw_b, 4096, 1024)  # same index, new weights
    for _ in range(2):
        check_gemv(g.matvec(3, x, 4096, 1024), raw_b, 12, 4096, 1024, x)
    X = m3.synth.activations(4096, seed=64, batch=5)  # larger staging buffers, batched path
    Y = g.matvec_batch(3, X, 4096, 1024)
    for b in range(5):
        check_gemv(Y[b], raw_b, 12, 4096, 1024, X[b])
    x2 = m3.synth.activations(4096, seed=65)  # back to one column, new x
    check_gemv(g.matvec(3, x2, 4096, 1024), raw_b, 12, 4096, 1024, x2)
    assert g.calls == 6
    m3.matvec_quant.set_tuning("offload_graph", 0)
    try:
        check_gemv(g.matvec(3, x2, 4096, 1024), raw_b, 12, 4096, 1024, x2)
    finally:
        m3.matvec_quant.set_tuning("offload_graph", 1)
    g.close()


def test_offload_mapped_and_copy_paths_agree(m3):
    """Batch-1 host calls on the tensor-core plan move x, y and the status word
    through mapped pinned memory; the copy-engine path (offload_mapped 0) and
    the non-tensor-core shapes keep the staged copies.  Same kernel, so the
    two paths give the same bits, and both match the oracle."""
    g = m3.inference_gpu.GpuOffload.try_new(4096, 2048)
    assert g is not None
    raw = m3.synth.weights(12, 4096, 2048, seed=71)
    raw_odd = m3.synth.weights(8, 4000, 100, seed=72)  # in_dim % 256 != 0: no tensor-core plan
    x = m3.synth.activations(4096, seed=73)
    xo = m3.synth.activations(4000, seed=74)
    assert g.upload(1, 12, raw, 4096, 2048) and g.upload(2, 8, raw_odd, 4000, 100)
    ys = {}
    for mapped in (1, 0, 1):
        m3.matvec_quant.set_tuning("offload_mapped", mapped)
        try:
            for _ in range(2):  # eager capture, then the replayed graph
                y = g.matvec(1, x, 4096, 2048)
                check_gemv(y, raw, 12, 4096, 2048, x)
                ys.setdefault(mapped, y.copy())
                assert np.array_equal(y.view(np.uint32), ys[mapped].view(np.uint32))
                check_gemv(g.matvec(2, xo, 4000, 100), raw_odd, 8, 4000, 100, xo)
        finally:
            m3.matvec_quant.set_tuning("offload_mapped", 1)
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))
    assert m3.matvec_quant.device_status(0) == 0
    g.close()


def test_offload_mapped_calls_across_batches_and_tensors(m3):
    """A mapped batch-1 call returns once its GEMV has published the call's
    sequence number, without synchronising the stream.  Interleave tensors,
    batch-1 calls (mapped), a batched call that regrows the staging buffers
    (restarting the sequence) and the tc8 kernel; every result must match the
    oracle and every call must return."""
    g = m3.inference_gpu.GpuOffload.try_new(4096, 4096)
    assert g is not None
    raws = {t: m3.synth.weights(12, 4096, 1000 + 700 * t, seed=80 + t) for t in (1, 2)}
    for t, r in raws.items():
        assert g.upload(t, 12, r, 4096, 1000 + 700 * t)
    xs = [m3.synth.activations(4096, seed=90 + i) for i in range(3)]
    plan = [(1, 1, 0), (2, 1, 0), (1, 1, 0), (2, 3, 0), (1, 1, 0), (2, 1, 1), (1, 1, 1), (2, 1, 0)]
    for t, batch, tc8 in plan:
        out = 1000 + 700 * t
        m3.matvec_quant.set_tuning("tc8", tc8)
        try:
            if batch == 1:
                check_gemv(g.matvec(t, xs[0], 4096, out), raws[t], 12, 4096, out, xs[0])
            else:
                Y = g.matvec_batch(t, np.stack(xs[:batch]), 4096, out)
                assert Y is not None
                for b in range(batch):
                    check_gemv(Y[b], raws[t], 12, 4096, out, xs[b])
        finally:
            m3.matvec_quant.set_tuning("tc8", 0)
    assert m3.matvec_quant.device_status(0) == 0
    g.close()
