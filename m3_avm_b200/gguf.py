"""GGUF ingest: read a GGUF file and upload its native blocks to the decode engine.

The reader follows the reference's parser (src/gguf.rs:73-157): magic
"GGUF" (either byte order), u32 version, u64 tensor and key counts, typed
key/values, tensor infos (name, dims innermost first, ggml dtype, offset),
tensor data starting at the header end rounded up to 32 bytes, each tensor at
data_offset + its offset.  The model shape comes from the keys
ModelConfig::from_gguf reads (src/inference.rs:37-89), the vocabulary size
from `<arch>.vocab_size` or else the length of `tokenizer.ggml.tokens`
(src/tokenizer.rs), the tensors by the llama names of LayerNames
(src/inference.rs:100-140); a missing output.weight falls back to the tied
token_embd.weight as in logits_from_head_cached.

Tensor bytes are read zero-copy through a numpy memmap and copied to HBM once
by `load_decoder` (the upload of `offload_gpu`, src/inference.rs:799).
``write_gguf`` writes the same layout (GGUF v3) for synthetic models.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from . import model, synth

GGUF_MAGIC = b"GGUF"
ALIGN = 32

# GGUF value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f", T_BOOL: "<?",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# bytes per block and elements per block of the tensor dtypes the engine takes
_DTYPE_BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 144), 14: (256, 210)}


@dataclass
class TensorInfo:
    name: str
    dims: list[int]   # innermost first (dims[0] = in_dim of a matrix)
    dtype: int
    offset: int       # within the data region
    n_elements: int

    def nbytes(self) -> int:
        be, bb = _DTYPE_BLOCK[self.dtype]
        if self.n_elements % be:
            raise ValueError(f"{self.name}: {self.n_elements} elements are not whole blocks of dtype {self.dtype}")
        return self.n_elements // be * bb


@dataclass
class GgufFile:
    path: str
    version: int
    kv: dict = field(default_factory=dict)
    tensors: list[TensorInfo] = field(default_factory=list)
    data_offset: int = 0
    _mm: np.ndarray | None = None

    def find(self, name: str) -> TensorInfo | None:
        for t in self.tensors:
            if t.name == name:
                return t
        return None

    def tensor_bytes(self, name: str) -> np.ndarray:
        """The tensor's raw bytes (a zero-copy view of the file)."""
        t = self.find(name)
        if t is None:
            raise KeyError(name)
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        start = self.data_offset + t.offset
        return self._mm[start:start + t.nbytes()]


class _Reader:
    def __init__(self, f):
        self.f = f

    def read(self, n: int) -> bytes:
        b = self.f.read(n)
        if len(b) != n:
            raise ValueError("truncated GGUF")
        return b

    def u32(self) -> int:
        return struct.unpack("<I", self.read(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.read(8))[0]

    def string(self) -> str:
        n = self.u64()
        if n > 10_000_000:
            raise ValueError(f"string length {n}")
        return self.read(n).decode("utf-8")

    def value(self, vtype: int):
        if vtype in _SCALAR:
            fmt = _SCALAR[vtype]
            return struct.unpack(fmt, self.read(struct.calcsize(fmt)))[0]
        if vtype == T_STR:
            return self.string()
        if vtype == T_ARR:
            at = self.u32()
            n = self.u64()
            return [self.value(at) for _ in range(n)]
        raise ValueError(f"GGUF value type {vtype}")


def read_gguf(path: str) -> GgufFile:
    with open(path, "rb") as f:
        r = _Reader(f)
        magic = r.read(4)
        if magic not in (GGUF_MAGIC, GGUF_MAGIC[::-1]):
            raise ValueError(f"not a GGUF file (magic {magic!r})")
        version = r.u32()
        n_tensors = r.u64()
        n_kv = r.u64()
        kv = {}
        for _ in range(n_kv):
            key = r.string()
            kv[key] = r.value(r.u32())
        tensors = []
        for _ in range(n_tensors):
            name = r.string()
            nd = r.u32()
            if nd > 8:
                raise ValueError(f"n_dims {nd}")
            dims = [r.u64() for _ in range(nd)]
            dtype = r.u32()
            off = r.u64()
            n = 1
            for d in dims:
                n *= d
            tensors.append(TensorInfo(name, dims, dtype, off, max(n, 1)))
        data_offset = (f.tell() + ALIGN - 1) // ALIGN * ALIGN
    return GgufFile(path, version, kv, tensors, data_offset)


def _pack_value(v) -> tuple[int, bytes]:
    if isinstance(v, bool):
        return T_BOOL, struct.pack("<?", v)
    if isinstance(v, int):
        return (T_U32, struct.pack("<I", v)) if 0 <= v < 2**32 else (T_I64, struct.pack("<q", v))
    if isinstance(v, float):
        return T_F32, struct.pack("<f", v)
    if isinstance(v, str):
        b = v.encode("utf-8")
        return T_STR, struct.pack("<Q", len(b)) + b
    if isinstance(v, list):
        if not v:
            return T_ARR, struct.pack("<IQ", T_U32, 0)
        at, _ = _pack_value(v[0])
        body = b"".join(_pack_value(x)[1] for x in v)
        return T_ARR, struct.pack("<IQ", at, len(v)) + body
    raise TypeError(type(v))


def write_gguf(path: str, kv: dict, tensors: list[tuple[str, list[int], int, np.ndarray]]) -> None:
    """GGUF v3: tensors = (name, dims innermost first, ggml dtype, bytes)."""
    head = bytearray()
    head += GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, v in kv.items():
        kb = k.encode("utf-8")
        vt, vb = _pack_value(v)
        head += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vt) + vb
    off = 0
    offsets = []
    for name, dims, dtype, arr in tensors:
        nb = name.encode("utf-8")
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", dtype, off)
        offsets.append(off)
        off += (np.asarray(arr).nbytes + ALIGN - 1) // ALIGN * ALIGN
    pad = (-len(head)) % ALIGN
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (_, _, _, arr), o in zip(tensors, offsets):
            b = np.ascontiguousarray(arr).view(np.uint8).tobytes()
            f.write(b + b"\0" * ((-len(b)) % ALIGN))


# ---------------------------------------------------------------- the model
_ARCH_PREFIXES = ("qwen2", "llama", "mistral")


def _get(kv: dict, keys, default):
    for k in keys:
        if k in kv:
            return kv[k]
    return default


def shape_from_gguf(g: GgufFile) -> model.LlamaShape:
    """ModelConfig::from_gguf restricted to the transformer families the engine runs."""
    kv = g.kv
    keys = lambda s: [f"{a}.{s}" for a in _ARCH_PREFIXES]  # noqa: E731
    hidden = int(_get(kv, keys("embedding_length") + ["general.embedding_length"], 2048))
    ffn = int(_get(kv, keys("feed_forward_length") + ["qwen2.intermediate_size"], 5632))
    n_layers = int(_get(kv, keys("block_count") + ["general.block_count"], 22))
    n_heads = int(_get(kv, keys("attention.head_count"), 32))
    n_kv = int(_get(kv, keys("attention.head_count_kv"), n_heads))
    vocab = int(_get(kv, ["qwen2.vocab_size", "llama.vocab_size", "general.vocab_size"], 32000))
    if vocab == 32000 and isinstance(kv.get("tokenizer.ggml.tokens"), list):
        vocab = len(kv["tokenizer.ggml.tokens"])
    theta = float(_get(kv, ["qwen2.rope.freq_base", "llama.rope.freq_base", "general.rope.freq_base"], 10000.0))

    def dt(name, default):
        t = g.find(name)
        return t.dtype if t is not None else default

    return model.LlamaShape(n_layers=n_layers, hidden=hidden, ffn=ffn, n_heads=n_heads, n_kv_heads=n_kv, vocab=vocab,
                            rope_theta=theta, embd_dtype=dt("token_embd.weight", 12),
                            attn_dtype=dt("blk.0.attn_q.weight", 12), gate_up_dtype=dt("blk.0.ffn_gate.weight", 12),
                            down_dtype=dt("blk.0.ffn_down.weight", 14),
                            head_dtype=dt("output.weight", dt("token_embd.weight", 14)))


def slot_names(shape: model.LlamaShape) -> dict[int, str]:
    names = {model.SLOT_EMBD: "token_embd.weight", model.SLOT_OUT_NORM: "output_norm.weight",
             model.SLOT_OUT: "output.weight"}
    for l in range(shape.n_layers):
        for kind, nm in enumerate(model.LAYER_NAMES):
            names[shape.slot(l, kind)] = f"blk.{l}.{nm}.weight"
    return names


def tensors_from_gguf(g: GgufFile, shape: model.LlamaShape) -> dict[int, tuple[np.ndarray, int]]:
    """slot -> (raw bytes view, dtype); output.weight falls back to token_embd.weight."""
    out = {}
    for slot, name in slot_names(shape).items():
        t = g.find(name)
        if t is None and slot == model.SLOT_OUT:
            name, t = "token_embd.weight", g.find("token_embd.weight")
        if t is None:
            raise KeyError(f"GGUF has no tensor {name}")
        out[slot] = (g.tensor_bytes(name), t.dtype)
    return out


def load_decoder(path: str, max_pos: int = 2048, device: int = 0, **kw):
    """Open a GGUF model and upload every tensor of the decode step once."""
    from .decoder import GpuDecoder

    g = read_gguf(path)
    shape = shape_from_gguf(g)
    dec = GpuDecoder(shape, max_pos=max_pos, device=device, **kw)
    dec.upload_all(tensors_from_gguf(g, shape))
    return dec, shape


def write_synthetic_model(path: str, shape: model.LlamaShape, seed: int) -> None:
    """A GGUF file of the synthetic model (llama keys, a placeholder token list
    whose length is the vocabulary, seeded blocks, f32 norms of ones)."""
    tens = model.synthetic_tensors(shape, seed)
    names = slot_names(shape)
    kv = {
        "general.architecture": "llama",
        "llama.block_count": shape.n_layers,
        "llama.embedding_length": shape.hidden,
        "llama.feed_forward_length": shape.ffn,
        "llama.attention.head_count": shape.n_heads,
        "llama.attention.head_count_kv": shape.n_kv_heads,
        "llama.rope.freq_base": float(shape.rope_theta),
        "llama.attention.layer_norm_rms_epsilon": 1e-5,
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(shape.vocab)],
    }
    entries = []
    for slot in sorted(tens):
        arr, dt = tens[slot]
        m = shape.matrix(slot)
        dims = [shape.hidden] if m is None else [m[1], m[2]]
        entries.append((names[slot], dims, dt, arr))
    write_gguf(path, kv, entries)


__all__ = ["GgufFile", "TensorInfo", "read_gguf", "write_gguf", "shape_from_gguf", "tensors_from_gguf",
           "load_decoder", "write_synthetic_model", "synth"]
