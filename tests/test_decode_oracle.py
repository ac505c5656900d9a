"""The CPU oracle of the decode step (RealInference::forward_one) on its own.

Pinned by the reference's unit tests of the pieces (src/inference.rs:1618-1641
RoPE identity and rotation, :1711-1717 GQA head order, :1777-1806 KV cache
growth and truncation, :1643-1658 greedy pick) and by an independent numpy
restatement of the whole step in float32, built from the oracle's bit-exact
block decoders (themselves pinned by the decoder known-answer tests).
"""
import numpy as np
import pytest

from oracle import oracle as O
from m3_avm_b200 import model, synth


def test_rope_identity_and_rotation():
    # src/inference.rs:1618-1641
    cs = O.rope_freqs(0, 4, 10000.0)
    assert np.allclose(O.apply_rope([1.0, 2.0, 3.0, 4.0], 1, 4, cs), [1, 2, 3, 4], atol=1e-6)
    w = O.apply_rope([1.0, 0.0, 3.0, 4.0], 1, 4, np.array([[0.0, 1.0], [1.0, 0.0]], np.float32))
    assert abs(w[0] + 3.0) < 1e-6 and abs(w[2] - 1.0) < 1e-6
    assert abs(w[1]) < 1e-6 and abs(w[3] - 4.0) < 1e-6
    assert abs(float(np.sum(w * w)) - 26.0) < 1e-5


def test_rope_freqs_arithmetic():
    # f = pos * theta^(-2i/hd) in f32, then (cos f, sin f)
    for pos in (0, 1, 7, 383):
        cs = O.rope_freqs(pos, 64, 500000.0)
        for i in (0, 1, 13, 31):
            f = pos * 500000.0 ** (-2.0 * i / 64.0)
            tol = 1e-6 + 4 * np.spacing(np.float32(f))  # f itself is rounded to f32 twice
            assert abs(cs[i, 0] - np.cos(f)) < tol
            assert abs(cs[i, 1] - np.sin(f)) < tol


def test_greedy_pick_rules():
    # src/inference.rs:1643-1658 (top_k = 1, no history): id 0 wins over 1.9
    assert O.greedy([2.0, 1.9]) == 0
    # ties go to the lowest index (stable descending sort)
    assert O.greedy([1.0, 3.0, 3.0, -1.0]) == 1
    assert O.greedy([-np.inf, -5.0]) == 1


def test_rms_norm_matches_formula():
    x = synth.activations(2048, 5)
    g = synth.activations(2048, 6)
    out = O.rms_norm(x, g)
    s = np.float32(0.0)
    for v in x:
        s = np.float32(s + np.float32(v * v))
    rms = np.sqrt(np.float32(s / np.float32(2048)) + np.float32(1e-5)).astype(np.float32)
    want = (x / rms).astype(np.float32) * g
    assert np.array_equal(out.view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_attention_head_matches_numpy():
    rng = np.random.default_rng(3)
    q = rng.standard_normal(64).astype(np.float32)
    k = rng.standard_normal((37, 64)).astype(np.float32)
    v = rng.standard_normal((37, 64)).astype(np.float32)
    out = O.attention_head(q, k, v)
    s = (k.astype(np.float64) @ q.astype(np.float64)) / 8.0
    w = np.exp(s - s.max())
    w /= w.sum()
    want = w @ v.astype(np.float64)
    assert np.max(np.abs(out - want)) < 1e-5 * np.max(np.abs(want)) + 1e-6


SMALL = model.LlamaShape(n_layers=2, hidden=256, ffn=512, n_heads=4, n_kv_heads=2, vocab=512, rope_theta=10000.0,
                         embd_dtype=12, attn_dtype=2, gate_up_dtype=8, down_dtype=14, head_dtype=14)


def numpy_forward(shape, T, tokens):
    """The step restated in numpy float32 with the oracle's exact decoders."""
    h, F, hd = shape.hidden, shape.ffn, shape.head_dim
    groups = shape.n_heads // shape.n_kv_heads

    def W(slot):
        arr, dt = T[slot]
        _, i, o = shape.matrix(slot)
        return O.dequantize(arr, dt, i * o).reshape(o, i)

    def norm(x, g):
        ms = np.float32(np.mean(x.astype(np.float64) ** 2))
        return (x / np.sqrt(ms + np.float32(1e-5))).astype(np.float32) * g

    def rope(v, nh, pos):
        cs = O.rope_freqs(pos, hd, shape.rope_theta)
        v = v.reshape(nh, hd).copy()
        a, b = v[:, : hd // 2].copy(), v[:, hd // 2:].copy()
        v[:, : hd // 2] = a * cs[:, 0] - b * cs[:, 1]
        v[:, hd // 2:] = a * cs[:, 1] + b * cs[:, 0]
        return v.reshape(-1)

    emb = W(model.SLOT_EMBD)
    head = W(model.SLOT_OUT)
    Ks = [[] for _ in range(shape.n_layers)]
    Vs = [[] for _ in range(shape.n_layers)]
    out = []
    for pos, tok in enumerate(tokens):
        x = emb[tok].copy()
        for l in range(shape.n_layers):
            s = lambda k: shape.slot(l, k)  # noqa: E731
            xn = norm(x, T[s(model.ATTN_NORM)][0])
            q = rope((W(s(model.ATTN_Q)) @ xn).astype(np.float32), shape.n_heads, pos)
            k = rope((W(s(model.ATTN_K)) @ xn).astype(np.float32), shape.n_kv_heads, pos)
            v = (W(s(model.ATTN_V)) @ xn).astype(np.float32)
            Ks[l].append(k)
            Vs[l].append(v)
            K, V = np.stack(Ks[l]), np.stack(Vs[l])
            att = np.zeros(h, np.float32)
            for hh in range(shape.n_heads):
                kv = hh // groups
                sc = K[:, kv * hd:(kv + 1) * hd] @ q[hh * hd:(hh + 1) * hd] / np.float32(np.sqrt(hd))
                w = np.exp(sc - sc.max())
                w /= w.sum()
                att[hh * hd:(hh + 1) * hd] = w @ V[:, kv * hd:(kv + 1) * hd]
            x = x + (W(s(model.ATTN_O)) @ att).astype(np.float32)
            xn = norm(x, T[s(model.FFN_NORM)][0])
            g = (W(s(model.FFN_GATE)) @ xn).astype(np.float32)
            u = (W(s(model.FFN_UP)) @ xn).astype(np.float32)
            with np.errstate(over="ignore"):
                hgu = g * (1.0 / (1.0 + np.exp(-g))) * u
            x = x + (W(s(model.FFN_DOWN)) @ hgu).astype(np.float32)
        out.append((head @ norm(x, T[model.SLOT_OUT_NORM][0])).astype(np.float32))
    return out


def test_oracle_step_matches_numpy_restatement():
    T = model.synthetic_tensors(SMALL, 4)
    toks = model.prompt_tokens(SMALL, 6, 8)
    dec = O.Decoder(SMALL.n_layers, SMALL.hidden, SMALL.ffn, SMALL.n_heads, SMALL.n_kv_heads, SMALL.vocab,
                    SMALL.rope_theta, 16, T)
    want = numpy_forward(SMALL, T, [int(t) for t in toks])
    for i, t in enumerate(toks):
        got = dec.forward(int(t))
        scale = float(np.max(np.abs(want[i])))
        assert np.max(np.abs(got - want[i])) <= 1e-4 * scale, (i, np.max(np.abs(got - want[i])), scale)
    assert dec.pos == len(toks)


def test_oracle_kv_cache_growth_and_truncate():
    # src/inference.rs:1777-1806: the cache grows one position per step,
    # truncation rolls back, and replaying the same token reproduces the step.
    T = model.synthetic_tensors(SMALL, 4)
    dec = O.Decoder(SMALL.n_layers, SMALL.hidden, SMALL.ffn, SMALL.n_heads, SMALL.n_kv_heads, SMALL.vocab,
                    SMALL.rope_theta, 8, T)
    a = dec.forward(1)
    b = dec.forward(2)
    assert dec.pos == 2
    dec.truncate(1)
    assert dec.pos == 1
    b2 = dec.forward(2)
    assert np.array_equal(b, b2)
    dec.reset()
    assert np.array_equal(dec.forward(1), a)


def test_oracle_rejects_bad_token_and_full_cache():
    T = model.synthetic_tensors(SMALL, 4)
    dec = O.Decoder(SMALL.n_layers, SMALL.hidden, SMALL.ffn, SMALL.n_heads, SMALL.n_kv_heads, SMALL.vocab,
                    SMALL.rope_theta, 2, T)
    with pytest.raises(ValueError):
        dec.forward(SMALL.vocab)
    dec.forward(0)
    dec.forward(0)
    with pytest.raises(ValueError):
        dec.forward(0)


def test_weight_bytes_per_token_of_the_1b_shape():
    # 16 x (q 2048^2 + k,v 512x2048 + o 2048^2 + gate,up 8192x2048 at 144 B/256;
    # down 2048x8192 at 210 B/256) + head 128256x2048 Q6_K + one Q4_K embedding row
    assert model.LLAMA_1B.weight_bytes_per_token() == 16 * 38535168 + 215470080 + 1152
