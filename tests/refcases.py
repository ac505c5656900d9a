"""Byte-level fixtures of the reference's own unit tests and benches, rebuilt here.

Each builder cites the m3_avm test it restates.  The activations use float32
arithmetic like the Rust tests (`(i as f32 * c).sin() * a`); their last ulp
may differ from Rust's libm, which only matters to tests that compare two
implementations on the same x, as these all do.
"""
from __future__ import annotations

import numpy as np


def _f32sin(n: int, c: float, a: float) -> np.ndarray:
    i = np.arange(n, dtype=np.float32)
    return (np.sin(i * np.float32(c)) * np.float32(a)).astype(np.float32)


def raw_q4k_ones(n: int) -> np.ndarray:
    """src/matvec_quant.rs:391-409: every element decodes to 1.0 (d=1, dmin=0, sc=1, m=0, q=1)."""
    assert n % 256 == 0
    raw = np.zeros((n // 256, 144), np.uint8)
    raw[:, 1] = 0x3C
    raw[:, 4:8] = 1
    raw[:, 12:16] = 1
    raw[:, 16:] = 0x11
    return raw.reshape(-1)


def q4k_pattern_37_11(in_dim: int, out_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:432-446 (and synth_q4k, src/bin/bench_gpu_gemv.rs:296-313)."""
    n = in_dim * out_dim
    raw = np.zeros((n // 256, 144), np.uint8)
    for b in range(n // 256):
        raw[b, 1] = 0x3C
        for i in range(12):
            raw[b, 4 + i] = (0x10 + ((b + i) & 0xFF) % 0x20) & 0xFF
        for i in range(128):
            raw[b, 16 + i] = ((b * 37) + (i * 11)) & 0xFF
    return raw.reshape(-1)


def synth_q4k(n: int) -> np.ndarray:
    """src/bin/bench_gpu_gemv.rs:296-313 (scales 0x10 + b + i, wrapping)."""
    raw = np.zeros((n // 256, 144), np.uint8)
    for b in range(n // 256):
        raw[b, 1] = 0x3C
        for i in range(12):
            raw[b, 4 + i] = (0x10 + b + i) & 0xFF
        for i in range(128):
            raw[b, 16 + i] = ((b * 37) + (i * 11)) & 0xFF
    return raw.reshape(-1)


def q4k_pattern_53_29(in_dim: int, out_dim: int, dmin_hi: int = 0x00) -> np.ndarray:
    """src/matvec_quant.rs:476-489 (dmin_hi=0xbc: dmin = -1.0) and :510-523 (dmin_hi=0)."""
    n = in_dim * out_dim
    raw = np.zeros((n // 256, 144), np.uint8)
    for b in range(n // 256):
        raw[b, 1] = 0x3C
        raw[b, 3] = dmin_hi
        for i in range(12):
            raw[b, 4 + i] = (0x10 + b + i) & 0xFF
        for i in range(128):
            raw[b, 16 + i] = ((b * 53) + (i * 29)) & 0xFF
    return raw.reshape(-1)


def synth_q6k(n: int) -> np.ndarray:
    """src/bin/bench_gpu_gemv.rs:316-336: d=1, alternating +1/-1 int8 scales."""
    raw = np.zeros((n // 256, 210), np.uint8)
    for b in range(n // 256):
        for i in range(128):
            raw[b, i] = ((b * 17) + (i * 7)) & 0xFF
        for i in range(64):
            raw[b, 128 + i] = ((b * 31) + (i * 3)) & 0xFF
        for i in range(16):
            raw[b, 192 + i] = 1 if (i + b) % 2 == 0 else 0xFF
        raw[b, 209] = 0x3C
    return raw.reshape(-1)


def q8_0_pattern(n: int) -> np.ndarray:
    """src/matvec_quant.rs:561-569: d=1, q = i - 16."""
    raw = np.zeros((n // 32, 34), np.uint8)
    raw[:, 1] = 0x3C
    raw[:, 2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    return raw.reshape(-1)


def x_ones_half(in_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:416: x[i] = (i + 1) * 0.5."""
    return ((np.arange(in_dim, dtype=np.float32) + 1) * np.float32(0.5)).astype(np.float32)


def x_sin(in_dim: int, c: float, a: float) -> np.ndarray:
    """x[i] = (i * c).sin() * a, as in src/matvec_quant.rs:447, :490, :524."""
    return _f32sin(in_dim, c, a)


def x_q8(in_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:570: x[i] = i * 0.3 + 1."""
    return (np.arange(in_dim, dtype=np.float32) * np.float32(0.3) + np.float32(1.0)).astype(np.float32)
