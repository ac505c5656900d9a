"""Fused dequantise-and-matvec with the API of m3_avm's src/matvec_quant.rs.

``matvec_quant`` keeps the reference's ``Option`` contract: ``None`` for an
unsupported dtype, zero dims, ``len(x) != in_dim`` or a short ``raw``; every
other call runs the sm_100a kernels of ``libm3gemv.so``.  Weights are GGUF
bytes with K = in_dim fastest: y[j] = sum_i x[i] * W[i + j*in_dim].
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib


def _u8(a) -> np.ndarray:
    if isinstance(a, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(a), np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8)


def quant_raw_len(dtype: int, n: int):
    """src/matvec_quant.rs:51-83: bytes for n elements, or None."""
    out = ctypes.c_uint64()
    rc = _lib.load().m3g_quant_raw_len(dtype, n, ctypes.byref(out))
    return out.value if rc == _lib.M3G_OK else None


def matvec_quant(x, raw, dtype: int, in_dim: int, out_dim: int):
    """src/matvec_quant.rs:87-109: Some(y) as a float32 array, or None."""
    xa = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    r = _u8(raw)
    # the reference's checks, in its order, before anything is allocated
    if xa.size != in_dim or in_dim == 0 or out_dim == 0:
        return None
    n = in_dim * out_dim
    if n >= 1 << 64:  # checked_mul overflows usize
        return None
    need = quant_raw_len(dtype, n)
    if need is None or r.size < need:
        return None
    y = np.empty(out_dim, np.float32)
    rc = _lib.load().m3g_matvec_quant(xa.ctypes.data, xa.size, r.ctypes.data, r.size, dtype, in_dim, out_dim,
                                      y.ctypes.data)
    if rc == _lib.M3G_ENONE:
        return None
    _lib.check(rc)
    return y[:out_dim]


def _direct(x, raw, dtype: int, in_dim: int, out_dim: int) -> np.ndarray:
    # The reference's direct kernels index raw without checks and panic on a
    # short slice; the mirror raises instead.
    y = matvec_quant(x, raw, dtype, in_dim, out_dim)
    if y is None:
        raise IndexError(_lib.last_error())
    return y


def matvec_q4k(x, raw, in_dim: int, out_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:221-223."""
    return _direct(x, raw, 12, in_dim, out_dim)


def matvec_q4k_impl(x, raw, in_dim: int, out_dim: int, use_avx2: bool) -> np.ndarray:
    """src/matvec_quant.rs:228-243; the SIMD selector has no meaning on the GPU."""
    del use_avx2
    return _direct(x, raw, 12, in_dim, out_dim)


def matvec_q6k(x, raw, in_dim: int, out_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:361-365."""
    return _direct(x, raw, 14, in_dim, out_dim)


def matvec_q4_0(x, raw, in_dim: int, out_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:368-372."""
    return _direct(x, raw, 2, in_dim, out_dim)


def matvec_q8_0(x, raw, in_dim: int, out_dim: int) -> np.ndarray:
    """src/matvec_quant.rs:375-382."""
    return _direct(x, raw, 8, in_dim, out_dim)


def matvec_quant_dev(x, raw, dtype: int, in_dim: int, out_dim: int, y=None, stream=None):
    """Device form over CUDA tensors: x is (in_dim,) or (batch, in_dim) float32,
    raw a uint8 tensor of GGUF bytes; returns y of shape (out_dim,) or (batch, out_dim)."""
    import torch

    batch = 1 if x.dim() == 1 else x.shape[0]
    if y is None:
        shape = (out_dim,) if x.dim() == 1 else (batch, out_dim)
        y = torch.empty(shape, dtype=torch.float32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    rc = _lib.load().m3g_matvec_quant_dev(x.data_ptr(), raw.data_ptr(), raw.numel(), dtype, in_dim, out_dim, batch,
                                          y.data_ptr(), ctypes.c_void_p(st))
    _lib.check(rc)
    return y


def set_tuning(key: str, value: int) -> None:
    _lib.check(_lib.load().m3g_set_tuning(key.encode(), int(value)))


def launch_count() -> int:
    return int(_lib.load().m3g_launch_count())


def device_status(device: int = 0, clear: bool = False) -> int:
    out = ctypes.c_uint32()
    _lib.check(_lib.load().m3g_device_status(device, ctypes.byref(out), int(clear)))
    return out.value


X_PLAIN, X_RMSNORM, X_SILU_MUL = 0, 1, 2


def matvec_fused_dev(x, raw, dtype: int, in_dim: int, out_dim: int, xmode: int = X_PLAIN, x2=None, gamma=None,
                     res=None, y=None, stream=None, swiglu: bool = False):
    """The decode step's fused GEMV over CUDA tensors (m3g_matvec_fused_dev):
    y = W x' (+ res), x' = x, rms_norm(x) * gamma, or silu(x) * x2; with
    swiglu, W is gate/up rows interleaved in blocks of 8 and y = silu(g) * u."""
    import torch

    if y is None:
        y = torch.empty(out_dim // 2 if swiglu else out_dim, dtype=torch.float32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    rc = _lib.load().m3g_matvec_fused_dev(x.data_ptr(), ptr(x2), ptr(gamma), ptr(res), xmode, 1 if swiglu else 0,
                                          raw.data_ptr(), raw.numel(), dtype, in_dim, out_dim, y.data_ptr(),
                                          ctypes.c_void_p(st))
    _lib.check(rc)
    return y


def matvec_fused_wait_dev(x, raw, dtype: int, in_dim: int, out_dim: int, ready, target: int, xmode: int = X_PLAIN,
                          x2=None, gamma=None, res=None, y=None, stream=None):
    """m3g_matvec_fused_wait_dev over CUDA tensors: the fused GEMV whose x
    preparation first waits (bounded by the tuning key peer_wait_us) until the
    device counter `ready` (an int32/uint32 tensor) reaches `target`."""
    import torch

    if y is None:
        y = torch.empty(out_dim, dtype=torch.float32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    rc = _lib.load().m3g_matvec_fused_wait_dev(x.data_ptr(), ptr(x2), ptr(gamma), ptr(res), xmode, raw.data_ptr(),
                                               raw.numel(), dtype, in_dim, out_dim, y.data_ptr(), ready.data_ptr(),
                                               int(target) & 0xFFFFFFFF, ctypes.c_void_p(st))
    _lib.check(rc)
    return y


def matvec_greedy_noalloc(x, raw, dtype: int, in_dim: int, out_dim: int, token=None, stream=None):
    """Greedy pick of W x into a device uint32 (m3g_matvec_greedy_noalloc): the
    library allocates nothing for it.  Returns the int32-typed token tensor."""
    import torch

    if token is None:
        token = torch.empty(1, dtype=torch.int32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    rc = _lib.load().m3g_matvec_greedy_noalloc(x.data_ptr(), raw.data_ptr(), raw.numel(), dtype, in_dim, out_dim,
                                               token.data_ptr(), ctypes.c_void_p(st))
    _lib.check(rc)
    return token
