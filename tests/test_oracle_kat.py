"""The CPU oracle against every known answer the reference's own tests hold.

Each test restates one unit test of m3_avm (file:line in its docstring) on the
oracle, plus a bit-exact cross-check of the decoders against the independent
ggml-format implementation in the `gguf` package.  These pin the oracle before
it is used to judge the GPU path.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests import refcases as R


# ---------------------------------------------------------------- src/quant.rs tests
def test_dequant_f32():
    """src/quant.rs:280-287."""
    src = bytes([0, 0, 128, 63, 0, 0, 0, 64])
    dst = O.dequantize(src, 0, 2)
    assert dst is not None
    assert abs(dst[0] - 1.0) < 1e-5 and abs(dst[1] - 2.0) < 1e-5


def test_dequant_q4_0_zero_block():
    """src/quant.rs:288-297: d=1.0, qs=0x88 -> all zeros."""
    src = bytearray(18)
    src[1] = 0x3C
    for i in range(2, 18):
        src[i] = 0x88
    dst = O.dequant_q4_0(src, 32)
    assert np.all(np.abs(dst) < 1e-5)


def test_dequant_q4_k_scales():
    """src/quant.rs:298-314: scales 0 -> 0; scales 0x10, qs 0x88 -> y[0] = 128."""
    src = bytearray(144)
    src[1] = 0x3C
    for i in range(16, 144):
        src[i] = 0x88
    dst = O.dequant_q4_k(src, 256)
    assert abs(dst[0]) < 1e-5
    for i in range(4, 16):
        src[i] = 0x10
    dst = O.dequant_q4_k(src, 256)
    assert abs(dst[0] - 128.0) < 1.0
    # The full vector that rule implies: sub-blocks 0-3 have sc = 16 (j < 4),
    # sub-blocks 4-7 have sc = (0x10 & 0xF) | (0x10 >> 6) << 4 = 0.
    assert np.all(dst[:128] == 128.0) and np.all(dst[128:] == 0.0)


def test_dequant_q6_k_signs():
    """src/quant.rs:315-370: zeros -> -32, int8 scale 0xFF -> +32, any bytes finite."""
    src = bytearray(210)
    src[209] = 0x3C
    for i in range(192, 208):
        src[i] = 1
    dst = O.dequant_q6_k(src, 256)
    assert np.all(np.isfinite(dst))
    assert abs(dst[0] + 32.0) < 0.1
    assert np.all(dst == -32.0)
    src3 = bytearray(210)
    src3[209] = 0x3C
    for i in range(192, 208):
        src3[i] = 0xFF
    dst3 = O.dequant_q6_k(src3, 256)
    assert abs(dst3[0] - 32.0) < 0.1
    src2 = bytearray(210)
    src2[209] = 0x3C
    for i in range(192, 208):
        src2[i] = 1
    for l in range(32):
        src2[l] = 0x22
        src2[l + 32] = 0x22
        src2[128 + l] = 0xAA
    dst2 = O.dequant_q6_k(src2, 256)
    assert np.all(np.isfinite(dst2))


def test_bf16_bits_rne():
    """src/quant.rs:371-391."""
    f = O.f32_to_bf16_bits
    assert f(1.0) == 0x3F80
    assert f(-2.5) == 0xC020
    assert f(0.0) == 0x0000
    assert f(math.inf) == 0x7F80
    assert f(-math.inf) == 0xFF80
    assert math.isnan(O.bf16_bits_to_f32(f(math.nan)))

    def fb(u):
        return float(np.array([u], np.uint32).view(np.float32)[0])

    assert f(fb(0x3F808000)) == 0x3F80
    assert f(fb(0x3F818000)) == 0x3F82
    assert f(fb(0x3F808001)) == 0x3F81
    assert f(fb(0x3F807FFF)) == 0x3F80
    for v in (1.0, -2.5, 0.5, 100.0, -0.0):
        back = O.bf16_bits_to_f32(f(v))
        assert back == v and math.copysign(1, back) == math.copysign(1, v)


def test_quantize_q4_0_roundtrip_bound():
    """src/quant.rs:392-426."""
    blk = O.quantize_q4_0([1.0] * 32)
    assert blk is not None
    back = O.dequant_q4_0(blk, 32)
    d = O.f16_to_f32(blk[0] | (blk[1] << 8))
    assert np.all(np.abs(back - 1.0) <= d / 2 + 1e-6)
    ramp = [(i - 16.0) * 0.5 for i in range(32)]
    blk2 = O.quantize_q4_0(ramp)
    back2 = O.dequant_q4_0(blk2, 32)
    d2 = O.f16_to_f32(blk2[0] | (blk2[1] << 8))
    assert np.all(np.abs(np.array(ramp, np.float32) - back2) <= d2 / 2 + 1e-4)
    zb = O.quantize_q4_0([0.0] * 32)
    assert np.all(O.dequant_q4_0(zb, 32) == 0.0)
    assert O.quantize_q4_0([1.0] * 31) is None
    bad = [1.0] * 32
    bad[3] = math.inf
    assert O.quantize_q4_0(bad) is None
    bad[3] = math.nan
    assert O.quantize_q4_0(bad) is None


def test_quantize_q8_0_roundtrip_bound():
    """src/quant.rs:427-448."""
    blk = O.quantize_q8_0([0.5] * 32)
    assert blk is not None
    back = O.dequantize(blk, 8, 32)
    d = O.f16_to_f32(blk[0] | (blk[1] << 8))
    assert np.all(np.abs(back - 0.5) <= d / 2 + 1e-6)
    assert O.quantize_q8_0([0.5] * 30) is None
    bad = [0.5] * 32
    bad[0] = -math.inf
    assert O.quantize_q8_0(bad) is None
    assert O.quant_block_info(4) == (32, 18)
    assert O.quant_block_info(8) == (32, 34)
    assert O.quant_block_info(12) is None
    assert O.quant_block_info(0) is None


def test_dequantize_dispatch_rules():
    """src/quant.rs:120-173: false cases, and dtype 13 decodes as Q4_K."""
    raw = R.synth_q4k(512)
    assert np.array_equal(O.dequantize(raw, 13, 512), O.dequantize(raw, 12, 512))
    assert O.dequantize(raw, 12, 100) is None            # n % 256
    assert O.dequantize(bytes(10), 14, 256) is None       # short Q6_K
    assert O.dequantize(bytes(10), 8, 32) is None         # short Q8_0
    assert O.dequantize(bytes(10), 3, 32) is None         # unknown dtype
    assert O.dequantize(bytes(2), 1, 2) is None           # short F16
    with pytest.raises(AssertionError):
        O.dequantize(bytes(10), 12, 256)                  # short Q4_K: the reference panics


# ---------------------------------------------------------------- src/matvec_quant.rs tests
def test_q4k_ones_matvec():
    """src/matvec_quant.rs:411-424: W of ones 16x16 -> y[j] = sum(x)."""
    x = R.x_ones_half(16)
    y = O.matvec_quant(x, R.raw_q4k_ones(256), 12, 16, 16)
    assert y is not None and y.shape == (16,)
    assert np.all(np.abs(y - x.sum()) < 1e-3)


def test_quant_matches_dequant_dot_q4k():
    """src/matvec_quant.rs:426-463: fused vs dequant + dense dot, 32x16 (blocks cross rows)."""
    raw = R.q4k_pattern_37_11(32, 16)
    x = R.x_sin(32, 0.13, 0.7)
    y = O.matvec_quant(x, raw, 12, 32, 16)
    w = O.dequantize(raw, 12, 512)
    y_ref = O.matvec_dense(x, w, 32, 16)
    assert np.max(np.abs(y - y_ref)) < 1e-2


def test_avx2_matches_scalar_q4k():
    """src/matvec_quant.rs:465-502: AVX2 kernel vs scalar parallel kernel, 256x16, dmin = -1."""
    raw = R.q4k_pattern_53_29(256, 16, dmin_hi=0xBC)
    x = R.x_sin(256, 0.31, 1.7)
    a = O.matvec_blocked(x, raw, 12, 256, 16)
    b = O.matvec_q4k_avx2(x, raw, 256, 16)
    max_ref = np.max(np.abs(a))
    assert max_ref > 1e-6
    assert np.max(np.abs(a - b)) / max_ref < 1e-4


def test_serial_matches_parallel_blocked():
    """src/matvec_quant.rs:503-532: serial vs parallel blocked loop, 48x32 (blocks cross rows)."""
    raw = R.q4k_pattern_53_29(48, 32)
    x = R.x_sin(48, 0.11, 0.9)
    a = O.matvec_blocked(x, raw, 12, 48, 32)
    b = O.matvec_blocked(x, raw, 12, 48, 32, serial=True)
    assert np.all(np.abs(a - b) < 1e-6)


def test_dispatcher_fallbacks():
    """src/matvec_quant.rs:533-553."""
    x8 = np.ones(8, np.float32)
    assert O.matvec_quant(x8, bytes(64), 0, 8, 2) is None
    assert O.matvec_quant(x8, bytes(10), 12, 32, 8) is None
    assert O.matvec_quant(x8, bytes(144), 12, 7, 5) is None
    raw = R.raw_q4k_ones(256)
    assert O.matvec_quant(np.ones(4, np.float32), raw, 12, 16, 16) is None
    x16 = np.full(16, 0.5, np.float32)
    a = O.matvec_quant(x16, raw, 12, 16, 16)
    b = O.matvec_q4k_impl(x16, raw, 16, 16, True)
    assert np.all(np.abs(a - b) < 1e-6)


def test_q8_0_matches_dequant():
    """src/matvec_quant.rs:555-581."""
    raw = R.q8_0_pattern(64)
    x = R.x_q8(8)
    y = O.matvec_quant(x, raw, 8, 8, 8)
    w = O.dequantize(raw, 8, 64)
    assert np.max(np.abs(y - O.matvec_dense(x, w, 8, 8))) < 1e-4


def test_gguf_orientation_nonsquare():
    """src/matvec.rs:101-120: W[i, j] = 10 i + j, x = 1 -> y[j] = 30 + 3 j."""
    in_dim, out_dim = 3, 4
    w = np.zeros(in_dim * out_dim, np.float32)
    for j in range(out_dim):
        for i in range(in_dim):
            w[i + j * in_dim] = i * 10 + j
    y = O.matvec_dense(np.ones(in_dim, np.float32), w, in_dim, out_dim)
    assert np.allclose(y, [30 + 3 * j for j in range(out_dim)], atol=1e-4)


# ---------------------------------------------------------------- independent ggml decoders
@pytest.mark.parametrize("dtype,name", [(2, "Q4_0"), (8, "Q8_0"), (12, "Q4_K"), (14, "Q6_K")])
def test_decoders_bit_exact_vs_gguf_package(dtype, name):
    """The oracle's decoders vs the `gguf` package's numpy ggml decoders, bit for bit."""
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType as T

    from m3_avm_b200 import synth

    n = 256 * 64
    raw = synth.weights(dtype, 256, 64, seed=1234 + dtype)
    mine = O.dequantize(raw, dtype, n)
    theirs = gq.dequantize(raw.reshape(-1, {2: 18, 8: 34, 12: 144, 14: 210}[dtype]), getattr(T, name)).reshape(-1)
    assert theirs.dtype == np.float32
    assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))
