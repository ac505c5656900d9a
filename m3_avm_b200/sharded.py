"""Row-sharded GEMV across the GPUs of one node (one process per GPU).

Rank r of `world` keeps output rows [r*RPR, min(out, (r+1)*RPR)) of each
tensor, RPR = ceil(out_dim / world); ``matvec`` computes the local rows and
every rank receives the full fp32 output: by one NCCL all-gather, or by peer
stores from the GEMV epilogue over NVLink (``exchange == "peer-stores"``)
where the ranks can map each other's exchange regions and the tuning key
``shard_p2p`` at creation asks for them (1; the default -1 from 8 ranks up,
where they measured faster).  This is the
multi-GPU form of the resident-weight offload (``inference_gpu.GpuOffload``);
the reference runs on one host CPU and has no counterpart.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib


def shard_plan(dtype: int, in_dim: int, out_dim: int, world: int, rank: int):
    """(row_begin, rows_local, rows_per_rank, byte_begin, byte_len) or None."""
    vals = [ctypes.c_uint64() for _ in range(5)]
    rc = _lib.load().m3g_shard_plan(dtype, in_dim, out_dim, world, rank, *[ctypes.byref(v) for v in vals])
    if rc == _lib.M3G_ENONE:
        return None
    _lib.check(rc)
    return tuple(v.value for v in vals)


def unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    _lib.check(_lib.load().m3g_shard_unique_id(ctypes.cast(buf, ctypes.c_void_p)))
    return bytes(buf)


class ShardedOffload:
    def __init__(self, device: int, rank: int, world: int, uid: bytes, max_in: int, max_out: int,
                 timeout_s: float = 60.0):
        if len(uid) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        self.device, self.rank, self.world = device, rank, world
        self.max_in, self.max_out = max_in, max_out
        idbuf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        h = ctypes.c_void_p()
        _lib.check(_lib.load().m3g_shard_create(device, rank, world, ctypes.cast(idbuf, ctypes.c_void_p), max_in,
                                                max_out, float(timeout_s), ctypes.byref(h)))
        self._h = h
        self._dims: dict[int, tuple[int, int, int]] = {}

    @classmethod
    def from_torch_dist(cls, device: int, max_in: int, max_out: int, timeout_s: float = 60.0):
        """Join using the ranks of an initialised torch.distributed group to share the id."""
        import torch.distributed as dist

        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(device, rank, world, obj[0], max_in, max_out, timeout_s)

    def upload(self, tidx: int, dtype: int, raw, in_dim: int, out_dim: int) -> bool:
        r = np.ascontiguousarray(np.frombuffer(bytes(raw), np.uint8) if isinstance(raw, (bytes, bytearray)) else raw,
                                 dtype=np.uint8)
        rc = _lib.load().m3g_shard_upload(self._h, tidx, dtype, r.ctypes.data, r.size, in_dim, out_dim)
        if rc == _lib.M3G_OK:
            self._dims[tidx] = (dtype, in_dim, out_dim)
        return rc == _lib.M3G_OK

    def info(self, tidx: int) -> tuple[int, int, int]:
        vals = [ctypes.c_uint64() for _ in range(3)]
        _lib.check(_lib.load().m3g_shard_info(self._h, tidx, *[ctypes.byref(v) for v in vals]))
        return tuple(v.value for v in vals)

    def matvec(self, tidx: int, x, in_dim: int, out_dim: int):
        """Host x (in_dim,) or (batch, in_dim) -> host y (batch, out_dim); every rank gets it all."""
        xa = np.ascontiguousarray(x, dtype=np.float32)
        batch = xa.shape[0] if xa.ndim == 2 else 1
        y = np.empty((batch, out_dim), np.float32)
        rc = _lib.load().m3g_shard_matvec(self._h, tidx, xa.ctypes.data, batch, in_dim, out_dim, y.ctypes.data)
        _lib.check(rc)
        return y if xa.ndim == 2 else y[0]

    def gather_len(self, tidx: int, batch: int = 1) -> int:
        _, _, rpr = self.info(tidx)
        return batch * rpr * self.world

    def matvec_dev(self, tidx: int, x, y, stream=None) -> None:
        """Device x (batch, in); y holds batch*RPR*world floats (see include/m3gemv.h)."""
        import torch

        batch = 1 if x.dim() == 1 else x.shape[0]
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(_lib.load().m3g_shard_matvec_dev(self._h, tidx, x.data_ptr(), batch, y.data_ptr(),
                                                    ctypes.c_void_p(st)))

    @property
    def calls(self) -> int:
        return int(_lib.load().m3g_shard_calls(self._h))

    @property
    def exchange(self) -> str:
        """'single' (one rank), 'nccl' (in-place all-gather) or 'peer-stores'
        (rows stored into every rank's region from the GEMV epilogue)."""
        return {0: "single", 1: "nccl", 2: "peer-stores"}.get(int(_lib.load().m3g_shard_exchange(self._h)), "?")

    def close(self) -> None:
        if self._h and self._h.value:
            _lib.load().m3g_shard_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
