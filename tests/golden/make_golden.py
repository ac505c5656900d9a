"""Generate tests/golden/golden_v1.npz: small fixed vectors for the GEMV path.

Each case holds GGUF bytes, an activation, the oracle's decoded weights and
the oracle's GEMV result (the reference-order fp32 computation, one thread,
so the values are deterministic).  The byte patterns are the reference's own
test fixtures (src/matvec_quant.rs:391-581, src/quant.rs:288-370,
src/bin/bench_gpu_gemv.rs:296-336) plus seeded synthetic tensors of every
dtype.  The oracle that produces them is pinned by the reference's
known-answer tests (tests/test_oracle_kat.py).

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from m3_avm_b200 import synth  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests import refcases as R  # noqa: E402

OUT = os.path.join(HERE, "golden_v1.npz")


def cases():
    yield "q4k_ones_16x16", 12, 16, 16, R.raw_q4k_ones(256), R.x_ones_half(16)
    yield "q4k_37_11_32x16", 12, 32, 16, R.q4k_pattern_37_11(32, 16), R.x_sin(32, 0.13, 0.7)
    yield "q4k_53_29_dminneg_256x16", 12, 256, 16, R.q4k_pattern_53_29(256, 16, 0xBC), R.x_sin(256, 0.31, 1.7)
    yield "q4k_53_29_48x32", 12, 48, 32, R.q4k_pattern_53_29(48, 32), R.x_sin(48, 0.11, 0.9)
    yield "q8_0_pattern_8x8", 8, 8, 8, R.q8_0_pattern(64), R.x_q8(8)
    yield "synth_q4k_1536x64", 12, 1536, 64, R.synth_q4k(1536 * 64), R.x_sin(1536, 0.017, 0.6)
    yield "synth_q6k_1536x64", 14, 1536, 64, R.synth_q6k(1536 * 64), R.x_sin(1536, 0.017, 0.6)
    for dtype, name in ((2, "q4_0"), (8, "q8_0"), (12, "q4k"), (14, "q6k")):
        for in_dim, out_dim in ((256, 40), (2048, 24)):
            yield (f"seeded_{name}_{in_dim}x{out_dim}", dtype, in_dim, out_dim,
                   synth.weights(dtype, in_dim, out_dim, seed=7 * in_dim + dtype),
                   synth.activations(in_dim, seed=in_dim + dtype))


def kat_blocks():
    """Decoder known answers (src/quant.rs:288-370) as (name, dtype, bytes, n)."""
    q40 = bytearray(18)
    q40[1] = 0x3C
    q40[2:] = b"\x88" * 16
    q4k = bytearray(144)
    q4k[1] = 0x3C
    q4k[16:] = b"\x88" * 128
    q4k[4:16] = b"\x10" * 12
    q6k_m32 = bytearray(210)
    q6k_m32[209] = 0x3C
    q6k_m32[192:208] = b"\x01" * 16
    q6k_p32 = bytearray(210)
    q6k_p32[209] = 0x3C
    q6k_p32[192:208] = b"\xff" * 16
    return [("kat_q4_0_zero", 2, bytes(q40), 32), ("kat_q4k_sc16", 12, bytes(q4k), 256),
            ("kat_q6k_minus32", 14, bytes(q6k_m32), 256), ("kat_q6k_plus32", 14, bytes(q6k_p32), 256)]


def main() -> None:
    arrays = {}
    names = []
    for name, dtype, in_dim, out_dim, raw, x in cases():
        raw = np.asarray(raw, np.uint8)
        x = np.asarray(x, np.float32)
        y = O.matvec_quant(x, raw, dtype, in_dim, out_dim, threads=1)
        w = O.dequantize(raw, dtype, in_dim * out_dim)
        assert y is not None and w is not None
        arrays[f"{name}/raw"] = raw
        arrays[f"{name}/x"] = x
        arrays[f"{name}/y"] = y
        if w.size <= 16384:
            arrays[f"{name}/w"] = w
        else:  # large decodes are kept as a CRC-32 of their f32 bytes
            arrays[f"{name}/wcrc"] = np.array([zlib.crc32(w.tobytes())], np.uint64)
        arrays[f"{name}/meta"] = np.array([dtype, in_dim, out_dim], np.int64)
        names.append(name)
    for name, dtype, raw, n in kat_blocks():
        arrays[f"{name}/raw"] = np.frombuffer(raw, np.uint8)
        arrays[f"{name}/w"] = O.dequantize(raw, dtype, n)
        arrays[f"{name}/meta"] = np.array([dtype, n, 1], np.int64)
        names.append(name)
    arrays["_names"] = np.array(names)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {len(names)} cases, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
