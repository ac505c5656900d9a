"""The C ABI library on a CPU-only machine: it loads, exports every declared
symbol, and its host-side rules agree with the oracle.  No GPU compute here."""
import ctypes
import math
import os
import re

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import HAS_CUDA, ROOT

HEADER = os.path.join(ROOT, "include", "m3gemv.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(m3g_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from m3_avm_b200 import _lib

    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from m3_avm_b200 import _lib

    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in m3gemv.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)
    assert lib.m3g_abi_version() == 1


def test_quant_raw_len_matches_oracle(lib):
    out = ctypes.c_uint64()
    for dtype in (0, 1, 2, 3, 8, 12, 13, 14, 15):
        for n in (0, 1, 31, 32, 64, 255, 256, 512, 4096 * 14336):
            rc = lib.m3g_quant_raw_len(dtype, n, ctypes.byref(out))
            want = O.quant_raw_len(dtype, n)
            if want is None:
                assert rc == -1
            else:
                assert rc == 0 and out.value == want


def test_bf16_helpers_match_oracle(lib):
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 1e3,
                           rng.integers(0, 2**32, 4000, dtype=np.uint64).astype(np.uint32).view(np.float32),
                           np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-45], np.float32)])
    for v in vals:
        a = lib.m3g_f32_to_bf16_bits(float(v))
        b = O.f32_to_bf16_bits(float(v))
        assert a == b, (v, hex(a), hex(b))
    for bits in range(0, 65536, 97):
        a = lib.m3g_bf16_bits_to_f32(bits)
        b = O.bf16_bits_to_f32(bits)
        assert (math.isnan(a) and math.isnan(b)) or a == b


def test_quantizers_match_oracle(lib):
    from m3_avm_b200 import quant

    rng = np.random.default_rng(11)
    cases = [rng.standard_normal(32).astype(np.float32) * s for s in (1e-9, 1e-3, 1.0, 300.0, 6e4)]
    cases += [np.zeros(32, np.float32), np.full(32, -1.0, np.float32),
              ((np.arange(32) - 16) * 0.5).astype(np.float32)]
    for c in cases:
        for fn, ofn, nb in ((quant.quantize_q4_0, O.quantize_q4_0, 18), (quant.quantize_q8_0, O.quantize_q8_0, 34)):
            dst = bytearray(nb)
            ok = fn(c, dst)
            want = ofn(c)
            assert ok == (want is not None)
            if ok:
                assert bytes(dst) == want
    bad = np.ones(32, np.float32)
    bad[5] = np.nan
    assert quant.quantize_q4_0(bad, bytearray(18)) is False
    assert quant.quantize_q8_0(np.ones(31, np.float32), bytearray(34)) is False
    assert quant.quant_block_info(4) == (32, 18) and quant.quant_block_info(12) is None


def test_python_mirror_none_rules_without_device():
    """The shape/dtype rules answer None before any device work."""
    from m3_avm_b200 import matvec_quant as M

    x8 = np.ones(8, np.float32)
    assert M.matvec_quant(x8, bytes(64), 0, 8, 2) is None
    assert M.matvec_quant(x8, bytes(10), 12, 32, 8) is None
    assert M.matvec_quant(x8, bytes(144), 12, 7, 5) is None
    assert M.matvec_quant(np.ones(4, np.float32), bytes(144), 12, 16, 16) is None
    # src/matvec_quant.rs:94-97: empty shapes and an overflowing in_dim * out_dim
    assert M.matvec_quant(np.zeros(0, np.float32), bytes(144), 12, 0, 16) is None
    assert M.matvec_quant(np.ones(256, np.float32), bytes(144), 12, 256, 0) is None
    assert M.matvec_quant(np.ones(256, np.float32), bytes(144), 12, 256, 2 ** 62) is None
    assert M.quant_raw_len(12, 512) == 288 and M.quant_raw_len(0, 512) is None


def test_c_abi_none_rules_without_device(lib):
    """The C entry point answers M3G_ENONE for empty shapes and an overflowing
    in_dim * out_dim before any device work (src/matvec_quant.rs:94-97)."""
    x = np.ones(256, np.float32)
    raw = np.zeros(144, np.uint8)
    y = np.zeros(4, np.float32)
    for in_dim, out_dim in [(0, 16), (256, 0), (256, 2 ** 62), (2 ** 40, 2 ** 40)]:
        rc = lib.m3g_matvec_quant(x.ctypes.data, min(in_dim, x.size), raw.ctypes.data, raw.size, 12, in_dim,
                                  out_dim, y.ctypes.data)
        assert rc == -1, (in_dim, out_dim, rc)
    assert np.all(y == 0)


@pytest.mark.skipif(HAS_CUDA, reason="checks the no-device error path")
def test_compute_fails_loudly_without_device(lib):
    """No CPU fallback: a valid compute call without a device returns M3G_ECUDA."""
    from m3_avm_b200 import matvec_quant as M
    from m3_avm_b200._lib import M3GError
    from tests import refcases as R

    with pytest.raises(M3GError):
        M.matvec_quant(np.ones(16, np.float32), R.raw_q4k_ones(256), 12, 16, 16)
    h = ctypes.c_void_p()
    assert lib.m3g_offload_create(0, 16, 16, ctypes.byref(h)) == -3
