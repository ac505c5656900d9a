"""GGUF block decoders and bf16/Q4_0/Q8_0 helpers with the API of m3_avm's src/quant.rs.

The decoders run on the GPU through ``libm3gemv.so`` and are bit-exact with
the reference.  Error behaviour mirrors the Rust functions: ``dequantize``
returns False where the reference does, and the fixed-type decoders raise
``AssertionError`` where the reference's ``assert!`` would panic.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

Q4_0_BLOCK_BYTES = 18
Q4_0_BLOCK_ELEMS = 32
Q8_0_BLOCK_BYTES = 34
Q8_0_BLOCK_ELEMS = 32


def _u8(a) -> np.ndarray:
    if isinstance(a, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(a), np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8)


def _decode(src, dtype: int, dst: np.ndarray, n: int) -> int:
    s = _u8(src)
    if dst.dtype != np.float32 or not dst.flags.c_contiguous or dst.size < n:
        raise ValueError("dst must be a contiguous float32 array with at least n elements")
    out = np.empty(n, np.float32)
    rc = _lib.load().m3g_dequantize(s.ctypes.data, s.size, dtype, out.ctypes.data, n)
    if rc == _lib.M3G_OK:
        dst[:n] = out
    return rc


def dequantize(src, dtype: int, dst: np.ndarray, n: int) -> bool:
    """src/quant.rs:120-173: decode n elements of ggml `dtype` into dst[:n]."""
    rc = _decode(src, dtype, dst, n)
    if rc == _lib.M3G_EPANIC:
        raise AssertionError(_lib.last_error())
    if rc in (_lib.M3G_OK, _lib.M3G_ENONE):
        return rc == _lib.M3G_OK
    raise _lib.M3GError(rc, _lib.last_error())


def _fixed(src, dtype: int, dst: np.ndarray, n: int, block: int) -> None:
    if n % block != 0:
        raise AssertionError(f"n % {block} != 0")
    rc = _decode(src, dtype, dst, n)
    if rc in (_lib.M3G_EPANIC, _lib.M3G_ENONE):
        raise AssertionError(_lib.last_error())
    _lib.check(rc)


def dequant_q4_0(src, dst: np.ndarray, n: int) -> None:
    """src/quant.rs:9-24."""
    _fixed(src, 2, dst, n, 32)


def dequant_q4_k(src, dst: np.ndarray, n: int) -> None:
    """src/quant.rs:41-71."""
    _fixed(src, 12, dst, n, 256)


def dequant_q6_k(src, dst: np.ndarray, n: int) -> None:
    """src/quant.rs:76-116."""
    _fixed(src, 14, dst, n, 256)


def f32_to_bf16_bits(x: float) -> int:
    """src/quant.rs:186-194."""
    return int(_lib.load().m3g_f32_to_bf16_bits(x))


def bf16_bits_to_f32(b: int) -> float:
    """src/quant.rs:197-199."""
    return float(_lib.load().m3g_bf16_bits_to_f32(b))


def _quantize(fn, src, nbytes: int, dst: bytearray | None):
    s = np.ascontiguousarray(src, dtype=np.float32)
    buf = np.zeros(max(nbytes, len(dst) if dst is not None else 0), np.uint8)
    rc = fn(s.ctypes.data, s.size, buf.ctypes.data, len(dst) if dst is not None else nbytes)
    if rc == _lib.M3G_ENONE:
        return False
    _lib.check(rc)
    if dst is not None:
        dst[: nbytes] = bytes(buf[:nbytes])
    return True


def quantize_q4_0(src, dst: bytearray) -> bool:
    """src/quant.rs:206-234: 32 floats -> one 18-byte Q4_0 block in dst."""
    return _quantize(_lib.load().m3g_quantize_q4_0, src, Q4_0_BLOCK_BYTES, dst)


def quantize_q8_0(src, dst: bytearray) -> bool:
    """src/quant.rs:239-264: 32 floats -> one 34-byte Q8_0 block in dst."""
    return _quantize(_lib.load().m3g_quantize_q8_0, src, Q8_0_BLOCK_BYTES, dst)


def quant_block_info(dtype: int):
    """src/quant.rs:269-275 (keyed by memory::DType numbering: 4 = Q4_0, 8 = Q8_0)."""
    if dtype == 4:
        return (Q4_0_BLOCK_ELEMS, Q4_0_BLOCK_BYTES)
    if dtype == 8:
        return (Q8_0_BLOCK_ELEMS, Q8_0_BLOCK_BYTES)
    return None


def dequantize_dev(src, dtype: int, n: int, out=None, stream=None):
    """Device form: src is a CUDA uint8 tensor; returns a CUDA float32 tensor of n elements."""
    import torch

    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=src.device)
    st = stream if stream is not None else torch.cuda.current_stream(src.device).cuda_stream
    rc = _lib.load().m3g_dequantize_dev(src.data_ptr(), src.numel(), dtype, out.data_ptr(), n, ctypes.c_void_p(st))
    _lib.check(rc)
    return out
