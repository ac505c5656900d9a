"""The VM's MATVEC and FFN opcodes on the device (exec_matvec,
src/vm.rs:2643-2685; exec_ffn, src/vm.rs:2471-2576), over CUDA tensors.

``exec_matvec(x, w, dtype, K, N)``: x of shape (K,) or (M, K), W the K*N
elements of a weight tensor (GGUF bytes or f32/f16).  M = 1 keeps the
reference's matvec orientation (y[j] = sum_i x[i] W[i + j*K], the fused
GEMV); M > 1 keeps its row-major [K, N] reading.  ``exec_ffn`` is
hidden = x W1 + b1, gated = hidden * sigmoid(hidden), out = gated W2 + b2
with the reference's bias rules.  Both raise M3GError where the opcode
returns an error.
"""
from __future__ import annotations

import ctypes

from . import _lib


def _stream(t, stream):
    import torch

    return stream if stream is not None else torch.cuda.current_stream(t.device).cuda_stream


def exec_matvec(x, w, dtype: int, K: int, N: int, y=None, stream=None):
    import torch

    M = 1 if x.dim() == 1 else x.shape[0]
    if x.shape[-1] != K:
        raise _lib.M3GError(_lib.M3G_EINVAL, f"MATVEC: x cols {x.shape[-1]} != W rows {K}")
    if y is None:
        y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    rc = _lib.load().m3g_vm_matvec_dev(x.data_ptr(), M, K, w.data_ptr(), w.numel() * w.element_size(), dtype, N,
                                       y.data_ptr(), ctypes.c_void_p(_stream(x, stream)))
    _lib.check(rc)
    return y


def exec_ffn(x, w1, dtype1: int, H: int, w2, dtype2: int, D_out: int, b1=None, b2=None, y=None, stream=None):
    import torch

    M, D = (1, x.shape[0]) if x.dim() == 1 else x.shape
    if y is None:
        y = torch.empty((M, D_out), dtype=torch.float32, device=x.device)
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    n = lambda t: t.numel() if t is not None else 0  # noqa: E731
    rc = _lib.load().m3g_vm_ffn_dev(x.data_ptr(), M, D, w1.data_ptr(), w1.numel() * w1.element_size(), dtype1, H,
                                    w2.data_ptr(), w2.numel() * w2.element_size(), dtype2, D_out, ptr(b1), n(b1),
                                    ptr(b2), n(b2), y.data_ptr(), ctypes.c_void_p(_stream(x, stream)))
    _lib.check(rc)
    return y
