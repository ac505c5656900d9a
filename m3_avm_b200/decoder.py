"""Device-resident greedy decode: the GPU form of RealInference's token loop.

``GpuDecoder`` mirrors the calls the reference's generation path makes on
RealInference (src/inference.rs): ``forward_one(token) -> logits``
(:953), ``prefill_logits(tokens) -> logits`` (:1388), greedy ``sample``
(``sample_with_params`` with top_k = 1, :1315), ``truncate_kv_cache`` and
``clear_kv_cache``.  ``generate`` runs the whole greedy loop on the device.
Every step runs on the CUDA library (``include/m3gemv.h``); there is no
host fallback, so a machine without the library or a GPU raises.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib, model


class GpuDecoder:
    """One engine per GPU.  With world > 1 the ranks (one process each) pass
    the same 128-byte NCCL id (``sharded.unique_id()``) and make the same calls
    in the same order; ffn_gate/up/down and the vocab head are row-sharded."""

    def __init__(self, shape: model.LlamaShape, max_pos: int = 1024, device: int = 0, rank: int = 0,
                 world: int = 1, nccl_id: bytes | None = None, timeout_s: float = 60.0):
        self.shape = shape
        self.max_pos = max_pos
        self.device = device
        self.rank, self.world = rank, world
        cfg = _lib.DecoderConfig(shape.n_layers, shape.hidden, shape.ffn, shape.n_heads, shape.n_kv_heads,
                                 shape.vocab, max_pos, shape.rope_theta)
        h = ctypes.c_void_p()
        if world == 1:
            rc = _lib.load().m3g_decoder_create(device, ctypes.byref(cfg), ctypes.byref(h))
        else:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("a sharded decoder needs the 128-byte NCCL unique id")
            idbuf = (ctypes.c_uint8 * 128).from_buffer_copy(nccl_id)
            rc = _lib.load().m3g_decoder_create_sharded(device, ctypes.byref(cfg), rank, world,
                                                        ctypes.cast(idbuf, ctypes.c_void_p), float(timeout_s),
                                                        ctypes.byref(h))
        _lib.check(rc)
        self._h = h

    @classmethod
    def from_torch_dist(cls, shape: model.LlamaShape, max_pos: int = 1024, device: int = 0, timeout_s: float = 60.0):
        """Join the ranks of an initialised torch.distributed group (rank 0's id is broadcast)."""
        import torch.distributed as dist

        from . import sharded

        rank, world = dist.get_rank(), dist.get_world_size()
        if world == 1:
            return cls(shape, max_pos, device)
        obj = [sharded.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(shape, max_pos, device, rank, world, obj[0], timeout_s)

    # ------------------------------------------------------------ weights
    def upload(self, slot: int, arr, dtype: int) -> None:
        a = np.ascontiguousarray(arr)
        _lib.check(_lib.load().m3g_decoder_upload(self._h, slot, dtype, a.ctypes.data, a.nbytes))

    def upload_all(self, tensors: dict[int, tuple[np.ndarray, int]]) -> None:
        for slot, (arr, dtype) in tensors.items():
            self.upload(slot, arr, dtype)

    @classmethod
    def synthetic(cls, shape: model.LlamaShape, seed: int, max_pos: int = 1024, device: int = 0):
        dec = cls(shape, max_pos, device)
        dec.upload_all(model.synthetic_tensors(shape, seed))
        return dec

    # ------------------------------------------------------------ the reference's calls
    def forward_one(self, token: int) -> np.ndarray:
        logits = np.empty(self.shape.vocab, np.float32)
        _lib.check(_lib.load().m3g_decoder_forward(self._h, int(token), logits.ctypes.data))
        return logits

    def prefill_logits(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.empty(self.shape.vocab, np.float32)
        if t.size == 0:
            return np.zeros(self.shape.vocab, np.float32)
        _lib.check(_lib.load().m3g_decoder_prefill(self._h, t.ctypes.data, t.size, logits.ctypes.data))
        return logits

    @staticmethod
    def sample(logits) -> int:
        """Greedy pick: the lowest index holding the largest logit."""
        la = np.asarray(logits, dtype=np.float32)
        return int(np.argmax(la)) if la.size else 0

    def generate(self, prompt, n_gen: int) -> np.ndarray:
        """Prefill `prompt` (may be empty to continue), then n_gen greedy tokens."""
        if len(prompt):
            t = np.ascontiguousarray(prompt, dtype=np.uint32)
            _lib.check(_lib.load().m3g_decoder_prefill(self._h, t.ctypes.data, t.size, None))
        out = np.empty(n_gen, np.uint32)
        if n_gen:
            _lib.check(_lib.load().m3g_decoder_generate(self._h, n_gen, out.ctypes.data))
        return out

    def run_async(self, n_steps: int) -> None:
        _lib.check(_lib.load().m3g_decoder_run_async(self._h, n_steps))

    def sync(self) -> None:
        _lib.check(_lib.load().m3g_decoder_sync(self._h))

    def tokens(self, first: int, n: int) -> np.ndarray:
        out = np.empty(n, np.uint32)
        _lib.check(_lib.load().m3g_decoder_tokens(self._h, first, n, out.ctypes.data))
        return out

    def truncate_kv_cache(self, n: int) -> None:
        _lib.check(_lib.load().m3g_decoder_truncate(self._h, n))

    def clear_kv_cache(self) -> None:
        self.truncate_kv_cache(0)

    def set_graph(self, use: bool) -> None:
        _lib.check(_lib.load().m3g_decoder_set_graph(self._h, 1 if use else 0))

    @property
    def pos(self) -> int:
        return int(_lib.load().m3g_decoder_pos(self._h))

    @property
    def stream(self) -> int:
        return int(_lib.load().m3g_decoder_stream(self._h) or 0)

    @property
    def exchange(self) -> str:
        """'single', 'nccl', 'peer-stores', 'head-only' (NCCL key all-reduce) or
        'head-only-peer' (peer key merge): how a sharded engine moves rows."""
        return {0: "single", 1: "nccl", 2: "peer-stores", 3: "head-only", 4: "head-only-peer"}.get(
            int(_lib.load().m3g_decoder_exchange(self._h)), "?")

    @property
    def logits_ptr(self) -> int:
        return int(_lib.load().m3g_decoder_logits_dev(self._h) or 0)

    def close(self) -> None:
        if self._h and self._h.value:
            _lib.load().m3g_decoder_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
