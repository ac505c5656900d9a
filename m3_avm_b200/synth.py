"""Seeded synthetic GGUF weights and activations (counter-based splitmix64).

Every value is a pure function of (seed, stream, index), so any slice of a
tensor can be regenerated independently and the same bytes feed the GPU
kernels and the CPU checks.  Distributions follow the benchmark workloads:

* Q4_K: d, dmin = fp16(|N(0, 0.02)|) (round-to-nearest-even), 12 scale bytes
  uniform in [0, 63], 128 quant bytes uniform (both nibbles uniform in [0, 15]).
* Q6_K: 128 ql and 64 qh bytes uniform, 16 int8 scales uniform in [-32, 31],
  d = fp16(|N(0, 0.02)|).
* Q8_0: d = fp16(|N(0, 0.02)|), 32 int8 quants uniform in [-127, 127].
* Q4_0: d = fp16(|N(0, 0.02)|), 16 quant bytes uniform.
* x: fp32 N(0, 1).
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_STREAM_MUL = np.uint64(0xD1B54A32D192ED03)

BLOCK = {12: (256, 144), 13: (256, 144), 14: (256, 210), 8: (32, 34), 2: (32, 18)}


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def u64(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """n 64-bit words of stream `stream` under `seed`, starting at counter `start`."""
    with np.errstate(over="ignore"):
        key = _mix(np.array([np.uint64(seed & (2**64 - 1)) ^ (np.uint64(stream) * _STREAM_MUL)], np.uint64))[0]
        idx = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        return _mix(key + idx * _GOLDEN)


def uniform01(seed: int, stream: int, n: int) -> np.ndarray:
    return (u64(seed, stream, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def normal(seed: int, stream: int, n: int) -> np.ndarray:
    """N(0, 1) in float64 by Box-Muller over two uniform streams."""
    u1 = 1.0 - uniform01(seed, stream, n)          # (0, 1]
    u2 = uniform01(seed, stream + 0x5151, n)
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def _f16_absnormal_bytes(seed: int, stream: int, n: int, sigma: float = 0.02) -> np.ndarray:
    v = np.abs(normal(seed, stream, n) * sigma).astype(np.float32).astype(np.float16)
    return v.view(np.uint8).reshape(n, 2)


def _bytes(seed: int, stream: int, n_rows: int, width: int) -> np.ndarray:
    words = (n_rows * width + 7) // 8
    return u64(seed, stream, words).view(np.uint8)[: n_rows * width].reshape(n_rows, width)


def q4k_blocks(n_blocks: int, seed: int) -> np.ndarray:
    out = np.empty((n_blocks, 144), np.uint8)
    out[:, 0:2] = _f16_absnormal_bytes(seed, 1, n_blocks)
    out[:, 2:4] = _f16_absnormal_bytes(seed, 2, n_blocks)
    out[:, 4:16] = _bytes(seed, 3, n_blocks, 12) & np.uint8(63)
    out[:, 16:144] = _bytes(seed, 4, n_blocks, 128)
    return out.reshape(-1)


def q6k_blocks(n_blocks: int, seed: int) -> np.ndarray:
    out = np.empty((n_blocks, 210), np.uint8)
    out[:, 0:128] = _bytes(seed, 5, n_blocks, 128)
    out[:, 128:192] = _bytes(seed, 6, n_blocks, 64)
    s = (_bytes(seed, 7, n_blocks, 16) & np.uint8(63)).astype(np.int16) - 32
    out[:, 192:208] = s.astype(np.int8).view(np.uint8)
    out[:, 208:210] = _f16_absnormal_bytes(seed, 8, n_blocks)
    return out.reshape(-1)


def q8_0_blocks(n_blocks: int, seed: int) -> np.ndarray:
    out = np.empty((n_blocks, 34), np.uint8)
    out[:, 0:2] = _f16_absnormal_bytes(seed, 9, n_blocks)
    h = _bytes(seed, 10, n_blocks, 64).view(np.uint16).astype(np.uint32)
    q = ((h * np.uint32(255)) >> np.uint32(16)).astype(np.int16) - 127
    out[:, 2:34] = q.astype(np.int8).view(np.uint8)
    return out.reshape(-1)


def q4_0_blocks(n_blocks: int, seed: int) -> np.ndarray:
    out = np.empty((n_blocks, 18), np.uint8)
    out[:, 0:2] = _f16_absnormal_bytes(seed, 11, n_blocks)
    out[:, 2:18] = _bytes(seed, 12, n_blocks, 16)
    return out.reshape(-1)


def weights(dtype: int, in_dim: int, out_dim: int, seed: int) -> np.ndarray:
    """GGUF bytes of an out_dim x in_dim tensor (K = in_dim fastest)."""
    be, _ = BLOCK[dtype]
    n = in_dim * out_dim
    if n % be:
        raise ValueError(f"{in_dim}x{out_dim} is not a whole number of {be}-element blocks")
    nb = n // be
    if dtype in (12, 13):
        return q4k_blocks(nb, seed)
    if dtype == 14:
        return q6k_blocks(nb, seed)
    if dtype == 8:
        return q8_0_blocks(nb, seed)
    if dtype == 2:
        return q4_0_blocks(nb, seed)
    raise ValueError(f"dtype {dtype}")


def activations(n: int, seed: int, batch: int | None = None) -> np.ndarray:
    """fp32 N(0, 1) activations: shape (n,) or (batch, n)."""
    count = n * (batch or 1)
    v = normal(seed, 13, count).astype(np.float32)
    return v if batch is None else v.reshape(batch, n)
