"""ctypes wrapper over the CPU oracle (``oracle/_build/liboracle.so``).

TEST INFRASTRUCTURE ONLY.  The oracle restates the reference's CPU algorithm
for the fused quantised GEMV path (src/quant.rs, src/matvec_quant.rs,
src/matvec.rs of m3_avm) so that the CUDA library can be checked against it.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module; the product never does.

Return conventions mirror the Rust API: ``None`` for ``Option::None``,
``AssertionError`` where the reference would panic on an ``assert!``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f64p = ctypes.POINTER(ctypes.c_double)
_sz = ctypes.c_size_t


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, strict IEEE flags)."""
    srcs = [os.path.join(_HERE, n) for n in ("m3q_oracle.c", "m3q_decode.c", "Makefile")]
    if force or not os.path.exists(_SO) or any(os.path.getmtime(_SO) < os.path.getmtime(s) for s in srcs):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_SO)
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f32_to_f16_bits.argtypes = [ctypes.c_float]
        L.or_f32_to_f16_bits.restype = ctypes.c_uint16
        L.or_f32_to_bf16_bits.argtypes = [ctypes.c_float]
        L.or_f32_to_bf16_bits.restype = ctypes.c_uint16
        L.or_bf16_bits_to_f32.argtypes = [ctypes.c_uint16]
        L.or_bf16_bits_to_f32.restype = ctypes.c_float
        for name in ("or_dequant_q4_0", "or_dequant_q4_k", "or_dequant_q6_k"):
            f = getattr(L, name)
            f.argtypes = [_u8p, _sz, _f32p, _sz]
            f.restype = ctypes.c_int
        L.or_dequantize.argtypes = [_u8p, _sz, ctypes.c_uint32, _f32p, _sz]
        L.or_dequantize.restype = ctypes.c_int
        L.or_get_scale_min_k4.argtypes = [ctypes.c_int, _u8p, _u8p, _u8p]
        L.or_get_scale_min_k4.restype = None
        for name in ("or_quantize_q4_0", "or_quantize_q8_0"):
            f = getattr(L, name)
            f.argtypes = [_f32p, _sz, _u8p, _sz]
            f.restype = ctypes.c_int
        L.or_quant_block_info.argtypes = [ctypes.c_uint32, ctypes.POINTER(_sz), ctypes.POINTER(_sz)]
        L.or_quant_block_info.restype = ctypes.c_int
        L.or_quant_raw_len.argtypes = [ctypes.c_uint32, _sz, ctypes.POINTER(_sz)]
        L.or_quant_raw_len.restype = ctypes.c_int
        L.or_matvec_q4k_avx2.argtypes = [_f32p, _u8p, _sz, _sz, _f32p, ctypes.c_int]
        L.or_matvec_q4k_avx2.restype = None
        L.or_matvec_q4k_impl.argtypes = [_f32p, _u8p, _sz, _sz, ctypes.c_int, _f32p, ctypes.c_int]
        L.or_matvec_q4k_impl.restype = None
        L.or_matvec_blocked.argtypes = [_f32p, _u8p, ctypes.c_uint32, _sz, _sz, _f32p, ctypes.c_int, ctypes.c_int]
        L.or_matvec_blocked.restype = None
        L.or_matvec_quant.argtypes = [_f32p, _sz, _u8p, _sz, ctypes.c_uint32, _sz, _sz, _f32p, ctypes.c_int]
        L.or_matvec_quant.restype = ctypes.c_int
        L.or_matvec_dense.argtypes = [_f32p, _f32p, _sz, _sz, _f32p]
        L.or_matvec_dense.restype = None
        L.or_row_l1.argtypes = [_u8p, _sz, ctypes.c_uint32, _sz, _sz, _f64p]
        L.or_row_l1.restype = ctypes.c_int
        L.or_max_threads.argtypes = []
        L.or_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(a), np.uint8) if isinstance(a, (bytes, bytearray)) else a, dtype=np.uint8)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, t):
    return a.ctypes.data_as(t)


def default_threads() -> int:
    return int(lib().or_max_threads())


# ---------------------------------------------------------------- scalars
def f16_to_f32(bits: int) -> float:
    return float(lib().or_f16_to_f32(bits))


def f32_to_f16_bits(x: float) -> int:
    return int(lib().or_f32_to_f16_bits(x))


def f32_to_bf16_bits(x: float) -> int:
    """src/quant.rs:186-194."""
    return int(lib().or_f32_to_bf16_bits(x))


def bf16_bits_to_f32(b: int) -> float:
    """src/quant.rs:197-199."""
    return float(lib().or_bf16_bits_to_f32(b))


# ---------------------------------------------------------------- decoders
def _dequant(fn, src, n: int) -> np.ndarray:
    s = _u8(src)
    dst = np.zeros(n, np.float32)
    rc = fn(_p(s, _u8p), s.size, _p(dst, _f32p), n)
    if rc < 0:
        raise AssertionError("reference assert! would fire (block count or source length)")
    return dst


def dequant_q4_0(src, n: int) -> np.ndarray:
    """src/quant.rs:9-24."""
    return _dequant(lib().or_dequant_q4_0, src, n)


def dequant_q4_k(src, n: int) -> np.ndarray:
    """src/quant.rs:41-71."""
    return _dequant(lib().or_dequant_q4_k, src, n)


def dequant_q6_k(src, n: int) -> np.ndarray:
    """src/quant.rs:76-116."""
    return _dequant(lib().or_dequant_q6_k, src, n)


def dequantize(src, dtype: int, n: int):
    """src/quant.rs:120-173: returns the f32 array, or None where it returns false."""
    s = _u8(src)
    dst = np.zeros(n, np.float32)
    rc = lib().or_dequantize(_p(s, _u8p), s.size, dtype, _p(dst, _f32p), n)
    if rc < 0:
        raise AssertionError("reference assert! would fire (block count or source length)")
    return dst if rc == 1 else None


def get_scale_min_k4(j: int, q) -> tuple[int, int]:
    """src/quant.rs:28-36."""
    qa = _u8(q)
    d = ctypes.c_uint8()
    m = ctypes.c_uint8()
    lib().or_get_scale_min_k4(j, _p(qa, _u8p), ctypes.byref(d), ctypes.byref(m))
    return d.value, m.value


def quantize_q4_0(src) -> bytes | None:
    """src/quant.rs:206-234."""
    s = _f32(src)
    dst = np.zeros(18, np.uint8)
    return bytes(dst) if lib().or_quantize_q4_0(_p(s, _f32p), s.size, _p(dst, _u8p), 18) else None


def quantize_q8_0(src) -> bytes | None:
    """src/quant.rs:239-264."""
    s = _f32(src)
    dst = np.zeros(34, np.uint8)
    return bytes(dst) if lib().or_quantize_q8_0(_p(s, _f32p), s.size, _p(dst, _u8p), 34) else None


def quant_block_info(dtype: int):
    """src/quant.rs:269-275."""
    e, b = _sz(), _sz()
    return (e.value, b.value) if lib().or_quant_block_info(dtype, ctypes.byref(e), ctypes.byref(b)) else None


# ---------------------------------------------------------------- fused GEMV
def quant_raw_len(dtype: int, n: int):
    """src/matvec_quant.rs:51-83."""
    out = _sz()
    return out.value if lib().or_quant_raw_len(dtype, n, ctypes.byref(out)) else None


def matvec_quant(x, raw, dtype: int, in_dim: int, out_dim: int, threads: int | None = None):
    """src/matvec_quant.rs:87-109 -> np.ndarray or None."""
    xa = _f32(x)
    r = _u8(raw)
    y = np.zeros(max(out_dim, 1), np.float32)
    ok = lib().or_matvec_quant(_p(xa, _f32p), xa.size, _p(r, _u8p), r.size, dtype, in_dim, out_dim,
                               _p(y, _f32p), threads or default_threads())
    return y[:out_dim] if ok else None


def matvec_q4k_impl(x, raw, in_dim: int, out_dim: int, use_avx2: bool, threads: int | None = None):
    """src/matvec_quant.rs:228-243."""
    xa, r = _f32(x), _u8(raw)
    y = np.zeros(out_dim, np.float32)
    lib().or_matvec_q4k_impl(_p(xa, _f32p), _p(r, _u8p), in_dim, out_dim, int(use_avx2), _p(y, _f32p),
                             threads or default_threads())
    return y


def matvec_q4k_avx2(x, raw, in_dim: int, out_dim: int, threads: int | None = None):
    """src/matvec_quant.rs:249-285 (no size gate)."""
    xa, r = _f32(x), _u8(raw)
    y = np.zeros(out_dim, np.float32)
    lib().or_matvec_q4k_avx2(_p(xa, _f32p), _p(r, _u8p), in_dim, out_dim, _p(y, _f32p), threads or default_threads())
    return y


def matvec_blocked(x, raw, dtype: int, in_dim: int, out_dim: int, serial: bool = False, threads: int | None = None):
    """src/matvec_quant.rs:124-216 (generic decode-then-dot loop)."""
    xa, r = _f32(x), _u8(raw)
    y = np.zeros(out_dim, np.float32)
    lib().or_matvec_blocked(_p(xa, _f32p), _p(r, _u8p), dtype, in_dim, out_dim, _p(y, _f32p),
                            threads or default_threads(), int(serial))
    return y


def matvec_dense(x, w, in_dim: int, out_dim: int):
    """src/matvec.rs:24-33, GGUF orientation y[j] = sum_i x[i] w[i + j*in]."""
    xa, wa = _f32(x), _f32(w)
    y = np.zeros(out_dim, np.float32)
    lib().or_matvec_dense(_p(xa, _f32p), _p(wa, _f32p), in_dim, out_dim, _p(y, _f32p))
    return y


def row_l1(raw, dtype: int, in_dim: int, out_dim: int) -> np.ndarray:
    """sum_i |w[i + j*in_dim]| per output row j, in float64."""
    r = _u8(raw)
    out = np.zeros(out_dim, np.float64)
    if not lib().or_row_l1(_p(r, _u8p), r.size, dtype, in_dim, out_dim, _p(out, _f64p)):
        raise ValueError("row_l1: cannot dequantise")
    return out


def gemv_bound(raw, dtype: int, in_dim: int, out_dim: int, x) -> np.ndarray:
    """Per-row tolerance 1e-5 * ||row||_1 * ||x||_inf (the GEMV parity bound)."""
    return 1e-5 * row_l1(raw, dtype, in_dim, out_dim) * float(np.max(np.abs(np.asarray(x, np.float64))))


# ---------------------------------------------------------------- decode step
def _bind_decoder(L) -> None:
    if getattr(L, "_decoder_bound", False):
        return
    vp = ctypes.c_void_p
    L.or_decoder_create.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_int]
    L.or_decoder_create.restype = vp
    L.or_decoder_destroy.argtypes = [vp]
    L.or_decoder_destroy.restype = None
    L.or_decoder_set.argtypes = [vp, ctypes.c_int, vp, _sz, ctypes.c_uint32]
    L.or_decoder_set.restype = ctypes.c_int
    L.or_decoder_forward.argtypes = [vp, ctypes.c_uint32, _f32p, ctypes.c_int]
    L.or_decoder_forward.restype = ctypes.c_int
    L.or_decoder_pos.argtypes = [vp]
    L.or_decoder_pos.restype = ctypes.c_int
    L.or_decoder_reset.argtypes = [vp]
    L.or_decoder_reset.restype = None
    L.or_decoder_truncate.argtypes = [vp, ctypes.c_int]
    L.or_decoder_truncate.restype = None
    L.or_rms_norm_into.argtypes = [_f32p, _f32p, _f32p, _sz]
    L.or_rms_norm_into.restype = None
    L.or_rope_freqs.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p]
    L.or_rope_freqs.restype = None
    L.or_apply_rope.argtypes = [_f32p, _sz, ctypes.c_int, ctypes.c_int, _f32p]
    L.or_apply_rope.restype = None
    L.or_greedy.argtypes = [_f32p, _sz]
    L.or_greedy.restype = ctypes.c_uint32
    L.or_attention_head.argtypes = [_f32p, _f32p, _f32p, _sz, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
    L.or_attention_head.restype = None
    L._decoder_bound = True


def rms_norm(x, gamma=None) -> np.ndarray:
    """rms_norm_into (src/inference.rs:1575-1585)."""
    L = lib()
    _bind_decoder(L)
    xa = _f32(x)
    out = np.zeros_like(xa)
    g = _f32(gamma) if gamma is not None else None
    L.or_rms_norm_into(_p(xa, _f32p), _p(g, _f32p) if g is not None else None, _p(out, _f32p), xa.size)
    return out


def rope_freqs(pos: int, head_dim: int, theta: float) -> np.ndarray:
    """(cos, sin) per pair for position `pos` (src/inference.rs:1000-1007), shape (head_dim/2, 2)."""
    L = lib()
    _bind_decoder(L)
    cs = np.zeros((max(head_dim, 2) // 2, 2), np.float32)
    L.or_rope_freqs(pos, head_dim, theta, _p(cs, _f32p))
    return cs


def apply_rope(v, n_heads: int, head_dim: int, cs) -> np.ndarray:
    """apply_rope (src/inference.rs:1554-1572) on a copy of v."""
    L = lib()
    _bind_decoder(L)
    out = _f32(v).copy()
    c = _f32(cs)
    L.or_apply_rope(_p(out, _f32p), out.size, n_heads, head_dim, _p(c, _f32p))
    return out


def greedy(logits) -> int:
    """sample_with_params with top_k = 1 (src/inference.rs:1315-1369)."""
    L = lib()
    _bind_decoder(L)
    la = _f32(logits)
    return int(L.or_greedy(_p(la, _f32p), la.size))


def attention_head(q, k_rows, v_rows) -> np.ndarray:
    """One head over npos cached rows (src/inference.rs:1052-1079)."""
    L = lib()
    _bind_decoder(L)
    qa, ka, va = _f32(q), _f32(k_rows), _f32(v_rows)
    npos, hd = ka.shape
    out = np.zeros(hd, np.float32)
    scores = np.zeros(max(npos, 1), np.float32)
    L.or_attention_head(_p(qa, _f32p), _p(ka, _f32p), _p(va, _f32p), hd, npos, hd, _p(out, _f32p), _p(scores, _f32p))
    return out


class Decoder:
    """RealInference::forward_one on the CPU (src/inference.rs:953-1152).

    ``tensors`` maps slot -> (uint8 or float32 array, ggml dtype); slots are
    0 token_embd, 1 output_norm, 2 output, then 9 per layer (attn_norm, q, k,
    v, o, ffn_norm, gate, up, down).  The arrays must outlive the decoder.
    """

    def __init__(self, n_layers, hidden, ffn, n_heads, n_kv_heads, vocab, rope_theta, max_pos, tensors,
                 threads: int | None = None):
        L = lib()
        _bind_decoder(L)
        self._L = L
        self.vocab = vocab
        self.threads = threads or default_threads()
        self._h = L.or_decoder_create(n_layers, hidden, ffn, n_heads, n_kv_heads, vocab, rope_theta, max_pos)
        if not self._h:
            raise ValueError("bad decoder shape")
        self._keep = []
        for slot, (arr, dtype) in tensors.items():
            a = np.ascontiguousarray(arr)
            self._keep.append(a)
            if not L.or_decoder_set(self._h, slot, a.ctypes.data, a.nbytes, dtype):
                raise ValueError(f"bad slot {slot}")

    def forward(self, token: int) -> np.ndarray:
        logits = np.zeros(self.vocab, np.float32)
        if not self._L.or_decoder_forward(self._h, token, _p(logits, _f32p), self.threads):
            raise ValueError("forward_one failed (missing tensor, bad token or full cache)")
        return logits

    @property
    def pos(self) -> int:
        return int(self._L.or_decoder_pos(self._h))

    def reset(self) -> None:
        self._L.or_decoder_reset(self._h)

    def truncate(self, n: int) -> None:
        self._L.or_decoder_truncate(self._h, n)

    def close(self) -> None:
        if self._h:
            self._L.or_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
