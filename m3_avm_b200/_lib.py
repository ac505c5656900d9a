"""ctypes binding of ``libm3gemv.so`` (the C ABI declared in ``include/m3gemv.h``).

The library is built in-tree by ``m3_avm_b200.build_lib``.  There is no
fallback: if the shared object is missing and cannot be built, importing
anything that needs it raises.
"""
from __future__ import annotations

import ctypes
import os

from . import build_lib

M3G_OK = 0
M3G_ENONE = -1
M3G_EINVAL = -2
M3G_ECUDA = -3
M3G_ENOMEM = -4
M3G_ENCCL = -5
M3G_ETIMEOUT = -6
M3G_ENOTFOUND = -7
M3G_EPANIC = -8

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32
_vp = ctypes.c_void_p



class DecoderConfig(ctypes.Structure):
    """m3g_decoder_config."""
    _fields_ = [("n_layers", _u64), ("hidden", _u64), ("ffn", _u64), ("n_heads", _u64), ("n_kv_heads", _u64),
                ("vocab", _u64), ("max_pos", _u64), ("rope_theta", ctypes.c_float)]


# name -> (restype, argtypes); the list every test checks against the header.
SIGNATURES: dict[str, tuple] = {
    "m3g_abi_version": (ctypes.c_int, []),
    "m3g_last_error": (ctypes.c_char_p, []),
    "m3g_quant_raw_len": (ctypes.c_int, [_u32, _u64, ctypes.POINTER(_u64)]),
    "m3g_f32_to_bf16_bits": (ctypes.c_uint16, [ctypes.c_float]),
    "m3g_bf16_bits_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
    "m3g_quantize_q4_0": (ctypes.c_int, [_vp, _u64, _vp, _u64]),
    "m3g_quantize_q8_0": (ctypes.c_int, [_vp, _u64, _vp, _u64]),
    "m3g_dequantize": (ctypes.c_int, [_vp, _u64, _u32, _vp, _u64]),
    "m3g_dequantize_dev": (ctypes.c_int, [_vp, _u64, _u32, _vp, _u64, _vp]),
    "m3g_matvec_quant": (ctypes.c_int, [_vp, _u64, _vp, _u64, _u32, _u64, _u64, _vp]),
    "m3g_matvec_quant_dev": (ctypes.c_int, [_vp, _vp, _u64, _u32, _u64, _u64, _u64, _vp, _vp]),
    "m3g_offload_create": (ctypes.c_int, [ctypes.c_int, _u64, _u64, ctypes.POINTER(_vp)]),
    "m3g_offload_upload": (ctypes.c_int, [_vp, _u64, _u32, _vp, _u64, _u64, _u64]),
    "m3g_offload_matvec": (ctypes.c_int, [_vp, _u64, _vp, _u64, _u64, _vp]),
    "m3g_offload_matvec_batch": (ctypes.c_int, [_vp, _u64, _vp, _u64, _u64, _u64, _vp]),
    "m3g_offload_matvec_dev": (ctypes.c_int, [_vp, _u64, _vp, _u64, _vp, _vp]),
    "m3g_offload_offloaded": (ctypes.c_int, [_vp, _u64]),
    "m3g_offload_tensor_count": (_u64, [_vp]),
    "m3g_offload_calls": (_u64, [_vp]),
    "m3g_offload_tensor_ptr": (_vp, [_vp, _u64]),
    "m3g_offload_destroy": (None, [_vp]),
    "m3g_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_u32), ctypes.c_int]),
    "m3g_launch_count": (_u64, []),
    "m3g_set_tuning": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int64]),
    "m3g_shard_plan": (ctypes.c_int, [_u32, _u64, _u64, ctypes.c_int, ctypes.c_int] + [ctypes.POINTER(_u64)] * 5),
    "m3g_shard_unique_id": (ctypes.c_int, [_vp]),
    "m3g_shard_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _u64, _u64, ctypes.c_double,
                                        ctypes.POINTER(_vp)]),
    "m3g_shard_upload": (ctypes.c_int, [_vp, _u64, _u32, _vp, _u64, _u64, _u64]),
    "m3g_shard_matvec_dev": (ctypes.c_int, [_vp, _u64, _vp, _u64, _vp, _vp]),
    "m3g_shard_matvec": (ctypes.c_int, [_vp, _u64, _vp, _u64, _u64, _u64, _vp]),
    "m3g_shard_info": (ctypes.c_int, [_vp, _u64] + [ctypes.POINTER(_u64)] * 3),
    "m3g_shard_calls": (_u64, [_vp]),
    "m3g_shard_exchange": (ctypes.c_int, [_vp]),
    "m3g_shard_destroy": (None, [_vp]),
    "m3g_matvec_fused_dev": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _u64, _u32, _u64,
                                            _u64, _vp, _vp]),
    "m3g_matvec_fused_wait_dev": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _u64, _u32, _u64, _u64,
                                                 _vp, _vp, _u32, _vp]),
    "m3g_decoder_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(DecoderConfig), ctypes.POINTER(_vp)]),
    "m3g_decoder_create_sharded": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(DecoderConfig), ctypes.c_int,
                                                  ctypes.c_int, _vp, ctypes.c_double, ctypes.POINTER(_vp)]),
    "m3g_decoder_upload": (ctypes.c_int, [_vp, _u32, _u32, _vp, _u64]),
    "m3g_decoder_forward": (ctypes.c_int, [_vp, _u32, _vp]),
    "m3g_decoder_prefill": (ctypes.c_int, [_vp, _vp, _u64, _vp]),
    "m3g_decoder_generate": (ctypes.c_int, [_vp, _u64, _vp]),
    "m3g_decoder_run_async": (ctypes.c_int, [_vp, _u64]),
    "m3g_decoder_sync": (ctypes.c_int, [_vp]),
    "m3g_decoder_tokens": (ctypes.c_int, [_vp, _u64, _u64, _vp]),
    "m3g_decoder_pos": (_u64, [_vp]),
    "m3g_decoder_truncate": (ctypes.c_int, [_vp, _u64]),
    "m3g_decoder_logits_dev": (_vp, [_vp]),
    "m3g_decoder_exchange": (ctypes.c_int, [_vp]),
    "m3g_decoder_stream": (_vp, [_vp]),
    "m3g_decoder_set_graph": (ctypes.c_int, [_vp, ctypes.c_int]),
    "m3g_decoder_destroy": (None, [_vp]),
    "m3g_matvec_greedy_noalloc": (ctypes.c_int, [_vp, _vp, _u64, _u32, _u64, _u64, _vp, _vp]),
    "m3g_vm_matvec_dev": (ctypes.c_int, [_vp, _u64, _u64, _vp, _u64, _u32, _u64, _vp, _vp]),
    "m3g_vm_ffn_dev": (ctypes.c_int, [_vp, _u64, _u64, _vp, _u64, _u32, _u64, _vp, _u64, _u32, _u64, _vp, _u64,
                                      _vp, _u64, _vp, _vp]),
}

_lib = None


def path() -> str:
    return build_lib.LIB


def load() -> ctypes.CDLL:
    """Load (building first if the sources are newer) and bind every symbol."""
    global _lib
    if _lib is not None:
        return _lib
    try:
        # The library links libnccl.so.2 by soname.  Loading torch first makes
        # both share torch's bundled NCCL; loading ours first would bind the
        # system copy and break a later `import torch`.
        import torch  # noqa: F401
    except ImportError:
        pass
    if not build_lib.up_to_date():
        try:
            build_lib.build()
        except Exception as exc:  # no nvcc on this machine and no prebuilt library
            if not os.path.exists(build_lib.LIB):
                raise ImportError(f"libm3gemv.so is missing and could not be built: {exc}") from exc
    L = ctypes.CDLL(build_lib.LIB)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class M3GError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"m3gemv error {code}: {msg}")
        self.code = code


def last_error() -> str:
    return (load().m3g_last_error() or b"").decode(errors="replace")


def check(rc: int) -> int:
    if rc != M3G_OK:
        raise M3GError(rc, last_error())
    return rc
