"""Shapes and seeded synthetic weights of the Llama-style models the decode
engine runs (the architecture RealInference::forward_one implements,
src/inference.rs:953-1152).

Tensor slots follow one fixed order shared by the device engine and the CPU
checks: 0 token_embd, 1 output_norm, 2 output (vocab head), then nine per
layer -- attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate,
ffn_up, ffn_down.  Quantised tensors are GGUF bytes in the GGUF orientation
(an out x in matrix, in fastest); norm weights are f32.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import synth

SLOT_EMBD, SLOT_OUT_NORM, SLOT_OUT, SLOT_LAYER0, SLOTS_PER_LAYER = 0, 1, 2, 3, 9
ATTN_NORM, ATTN_Q, ATTN_K, ATTN_V, ATTN_O, FFN_NORM, FFN_GATE, FFN_UP, FFN_DOWN = range(9)
LAYER_NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
               "ffn_down")


@dataclass(frozen=True)
class LlamaShape:
    n_layers: int = 16
    hidden: int = 2048
    ffn: int = 8192
    n_heads: int = 32
    n_kv_heads: int = 8
    vocab: int = 128256
    rope_theta: float = 500000.0
    # ggml dtypes of the Q4_K_M mix: Q4_K attention, gate/up and embedding,
    # Q6_K ffn_down and output.
    embd_dtype: int = 12
    attn_dtype: int = 12
    gate_up_dtype: int = 12
    down_dtype: int = 14
    head_dtype: int = 14

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def slot(self, layer: int, kind: int) -> int:
        return SLOT_LAYER0 + SLOTS_PER_LAYER * layer + kind

    def n_slots(self) -> int:
        return SLOT_LAYER0 + SLOTS_PER_LAYER * self.n_layers

    def matrix(self, slot: int) -> tuple[int, int, int] | None:
        """(dtype, in_dim, out_dim) of a quantised slot, None for a norm."""
        h, F, kv = self.hidden, self.ffn, self.kv_dim
        if slot == SLOT_EMBD:
            return self.embd_dtype, h, self.vocab
        if slot == SLOT_OUT:
            return self.head_dtype, h, self.vocab
        if slot == SLOT_OUT_NORM:
            return None
        kind = (slot - SLOT_LAYER0) % SLOTS_PER_LAYER
        return {
            ATTN_NORM: None, FFN_NORM: None,
            ATTN_Q: (self.attn_dtype, h, h), ATTN_K: (self.attn_dtype, h, kv), ATTN_V: (self.attn_dtype, h, kv),
            ATTN_O: (self.attn_dtype, h, h), FFN_GATE: (self.gate_up_dtype, h, F),
            FFN_UP: (self.gate_up_dtype, h, F), FFN_DOWN: (self.down_dtype, F, h),
        }[kind]

    def weight_bytes_per_token(self) -> int:
        """Bytes of every matrix one decode step streams (all layers + head; the
        embedding contributes one row)."""
        total = 0
        for s in range(self.n_slots()):
            m = self.matrix(s)
            if m is None or s == SLOT_EMBD:
                continue
            dt, i, o = m
            be, bb = synth.BLOCK[dt]
            total += i * o // be * bb
        be, bb = synth.BLOCK[self.embd_dtype]
        return total + self.hidden // be * bb


LLAMA_1B = LlamaShape()


def synthetic_tensors(shape: LlamaShape, seed: int) -> dict[int, tuple[np.ndarray, int]]:
    """slot -> (array, ggml dtype): seeded GGUF blocks for every matrix (each
    slot its own seed), f32 ones for every norm."""
    out: dict[int, tuple[np.ndarray, int]] = {}
    for s in range(shape.n_slots()):
        m = shape.matrix(s)
        if m is None:
            out[s] = (np.ones(shape.hidden, np.float32), 0)
        else:
            dt, i, o = m
            out[s] = (synth.weights(dt, i, o, seed * 1000003 + s), dt)
    return out


def prompt_tokens(shape: LlamaShape, n: int, seed: int) -> np.ndarray:
    """n token ids uniform in [0, vocab)."""
    return (synth.u64(seed, 77, n) % np.uint64(shape.vocab)).astype(np.uint32)
