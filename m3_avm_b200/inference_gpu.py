"""Resident-weight GEMV offload with the shape of m3_avm's GpuOffload (src/inference_gpu.rs).

Weights are uploaded once, in their native GGUF block layout, and stay in
HBM; each ``matvec`` moves only x and y.  As in the reference, failures never
propagate: ``try_new`` returns None without a device, ``upload`` returns
False for a tensor the kernels cannot serve, and ``matvec`` returns None so
the caller can take another route.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib


class GpuOffload:
    def __init__(self, handle: int, device: int, max_in: int, max_out: int):
        self._h = ctypes.c_void_p(handle)
        self.device = device
        self.max_in = max_in
        self.max_out = max_out
        self.head = None  # tensor index of the LM head, if offloaded (src/inference_gpu.rs:51-52)

    @classmethod
    def try_new(cls, max_in: int, max_out: int, device: int = 0):
        """src/inference_gpu.rs:58-127: None when no device is usable."""
        h = ctypes.c_void_p()
        rc = _lib.load().m3g_offload_create(device, max_in, max_out, ctypes.byref(h))
        if rc != _lib.M3G_OK or not h.value:
            return None
        return cls(h.value, device, max_in, max_out)

    def upload(self, tidx: int, dtype: int, raw, in_dim: int, out_dim: int) -> bool:
        """src/inference_gpu.rs:131-177."""
        r = raw if isinstance(raw, np.ndarray) else np.frombuffer(bytes(raw), np.uint8)
        r = np.ascontiguousarray(r, dtype=np.uint8)
        rc = _lib.load().m3g_offload_upload(self._h, tidx, dtype, r.ctypes.data, r.size, in_dim, out_dim)
        return rc == _lib.M3G_OK

    def offloaded(self, tidx: int) -> bool:
        return bool(_lib.load().m3g_offload_offloaded(self._h, tidx))

    def tensor_count(self) -> int:
        return int(_lib.load().m3g_offload_tensor_count(self._h))

    @property
    def calls(self) -> int:
        return int(_lib.load().m3g_offload_calls(self._h))

    def matvec(self, tidx: int, x, in_dim: int, out_dim: int, out=None):
        """src/inference_gpu.rs:188-237: y as float32, or None.  `out` (a
        C-contiguous float32 array of out_dim values) receives y instead of a
        new array, so a caller's token loop allocates nothing per call."""
        xa = x if (isinstance(x, np.ndarray) and x.dtype == np.float32 and x.flags.c_contiguous) else \
            np.ascontiguousarray(x, dtype=np.float32)
        if xa.size != in_dim:
            return None
        if out is None:
            y = np.empty(out_dim, np.float32)
        else:
            if out.dtype != np.float32 or out.size != out_dim or not out.flags.c_contiguous:
                raise ValueError("out must be a C-contiguous float32 array of out_dim values")
            y = out
        rc = _lib.load().m3g_offload_matvec(self._h, tidx, xa.ctypes.data, in_dim, out_dim, y.ctypes.data)
        return y if rc == _lib.M3G_OK else None

    def matvec_batch(self, tidx: int, x, in_dim: int, out_dim: int):
        xa = np.ascontiguousarray(x, dtype=np.float32)
        batch = xa.shape[0] if xa.ndim == 2 else 1
        y = np.empty((batch, out_dim), np.float32)
        rc = _lib.load().m3g_offload_matvec_batch(self._h, tidx, xa.ctypes.data, batch, in_dim, out_dim,
                                                  y.ctypes.data)
        return y if rc == _lib.M3G_OK else None

    def matvec_dev(self, tidx: int, x, y, stream=None) -> None:
        """x (batch, in) / y (batch, out) CUDA float32 tensors; enqueued, not synchronised."""
        import torch

        batch = 1 if x.dim() == 1 else x.shape[0]
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(_lib.load().m3g_offload_matvec_dev(self._h, tidx, x.data_ptr(), batch, y.data_ptr(),
                                                      ctypes.c_void_p(st)))

    def tensor_ptr(self, tidx: int) -> int:
        return int(_lib.load().m3g_offload_tensor_ptr(self._h, tidx) or 0)

    def close(self) -> None:
        if self._h and self._h.value:
            _lib.load().m3g_offload_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
