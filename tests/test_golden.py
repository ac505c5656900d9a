"""Committed golden vectors (tests/golden/golden_v1.npz) against the oracle
(CPU) and against the GPU kernels (marked gpu)."""
import os
import zlib

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_v1.npz")


def load():
    z = np.load(GOLDEN)
    out = {}
    for name in z["_names"]:
        name = str(name)
        out[name] = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return out


CASES = load()
GEMV = [n for n, c in CASES.items() if "y" in c]


def decoded_matches(w, c):
    if "w" in c:
        return np.array_equal(w.view(np.uint32), c["w"].view(np.uint32))
    return zlib.crc32(np.ascontiguousarray(w, np.float32).tobytes()) == int(c["wcrc"][0])


def row_l1(c, dtype, a, b):
    w = O.dequantize(c["raw"], dtype, a * b)
    return np.abs(w.astype(np.float64)).reshape(b, a).sum(1)


def test_reference_known_answers_in_fixture():
    """The fixture itself carries the values the reference's tests assert."""
    assert np.all(CASES["kat_q4_0_zero"]["w"] == 0.0)
    assert CASES["kat_q4k_sc16"]["w"][0] == 128.0
    assert np.all(CASES["kat_q6k_minus32"]["w"] == -32.0)
    assert np.all(CASES["kat_q6k_plus32"]["w"] == 32.0)
    c = CASES["q4k_ones_16x16"]
    assert np.all(np.abs(c["y"] - c["x"].sum()) < 1e-3)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_reproduces_golden(name):
    c = CASES[name]
    dtype, a, b = (int(v) for v in c["meta"])
    if "y" in c:
        w = O.dequantize(c["raw"], dtype, a * b)
        assert decoded_matches(w, c)
        y = O.matvec_quant(c["x"], c["raw"], dtype, a, b, threads=1)
        assert np.array_equal(y.view(np.uint32), c["y"].view(np.uint32))
    else:
        w = O.dequantize(c["raw"], dtype, a)
        assert np.array_equal(w.view(np.uint32), c["w"].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_matches_golden(name):
    from m3_avm_b200 import matvec_quant, quant

    c = CASES[name]
    dtype, a, b = (int(v) for v in c["meta"])
    n = a * b if "y" in c else a
    w = np.zeros(n, np.float32)
    assert quant.dequantize(c["raw"], dtype, w, n)
    assert decoded_matches(w, c)
    if "y" in c:
        y = matvec_quant.matvec_quant(c["x"], c["raw"], dtype, a, b)
        bound = 1e-5 * row_l1(c, dtype, a, b) * np.abs(c["x"]).max() + 1e-30
        assert np.all(np.abs(y.astype(np.float64) - c["y"]) <= bound)
