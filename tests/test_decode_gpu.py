"""GPU parity of the device decode engine against the CPU oracle of
RealInference::forward_one (src/inference.rs:953-1152).

* the fused GEMV forms (norm input, SwiGLU input, residual epilogue), each
  row within the GEMV bound 1e-5 * ||row||_1 * ||x'||_inf of the oracle;
* whole decode steps, teacher-forced (both sides fed the same tokens): the
  logits of every step within DECODE_TOL * ||logits||_inf of the oracle, and
  the greedy picks equal wherever the oracle's top-2 gap exceeds twice the
  observed error (near-tied logits of a random-weight model may pick either);
* the device token loop: generate() equals the host-driven forward_one loop,
  graph replay equals eager launches bit for bit, truncation replays a step
  bit for bit, and the engine's failure rules.
"""
import numpy as np
import pytest

from oracle import oracle as O
from m3_avm_b200 import model, synth

pytestmark = pytest.mark.gpu

# Relative logit tolerance of a teacher-forced step.  Each step chains
# 7 * n_layers + 1 GEMVs (each within its 1e-5 bound, typically ~1e-7),
# softmaxes and norms; a max error of 1e-4 of the logit scale leaves a wide
# margin over the errors observed at these shapes.
DECODE_TOL = 1e-4

# Zero-mean formats (Q4_0, Q8_0, Q6_K) keep activations of a random model
# well-conditioned, so attention is not one-hot and every kernel is exercised.
WELL = model.LlamaShape(n_layers=2, hidden=2048, ffn=2048, n_heads=32, n_kv_heads=8, vocab=4096,
                        rope_theta=500000.0, embd_dtype=12, attn_dtype=2, gate_up_dtype=8, down_dtype=14,
                        head_dtype=14)
# head_dim 128 and mixed dtypes inside q/k/v and gate/up (launched separately).
HD128 = model.LlamaShape(n_layers=2, hidden=2048, ffn=4096, n_heads=16, n_kv_heads=4, vocab=2048,
                         rope_theta=10000.0, embd_dtype=14, attn_dtype=12, gate_up_dtype=12, down_dtype=14,
                         head_dtype=12)


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    from m3_avm_b200 import _lib

    _lib.load()
    return torch


def mixed_tensors(shape, seed):
    """synthetic_tensors with k and up switched to Q8_0 so the concatenation
    falls back to separate launches."""
    T = model.synthetic_tensors(shape, seed)
    for l in range(shape.n_layers):
        for kind in (model.ATTN_K, model.FFN_UP):
            s = shape.slot(l, kind)
            _, i, o = shape.matrix(s)
            T[s] = (synth.weights(8, i, o, seed * 31 + s), 8)
    return T


def oracle_decoder(shape, T, max_pos):
    return O.Decoder(shape.n_layers, shape.hidden, shape.ffn, shape.n_heads, shape.n_kv_heads, shape.vocab,
                     shape.rope_theta, max_pos, T)


def gpu_decoder(shape, T, max_pos):
    from m3_avm_b200.decoder import GpuDecoder

    d = GpuDecoder(shape, max_pos=max_pos)
    d.upload_all(T)
    return d


def teacher_forced(shape, T, tokens, max_pos=64):
    g = gpu_decoder(shape, T, max_pos)
    o = oracle_decoder(shape, T, max_pos)
    worst = 0.0
    for i, t in enumerate(tokens):
        lg = g.forward_one(int(t))
        lo = o.forward(int(t))
        assert np.all(np.isfinite(lg))
        scale = float(np.max(np.abs(lo)))
        err = float(np.max(np.abs(lg.astype(np.float64) - lo)))
        worst = max(worst, err / scale)
        assert err <= DECODE_TOL * scale, f"step {i}: max err {err:.3g} vs logit scale {scale:.3g}"
        top = np.sort(lo)[::-1]
        if top[0] - top[1] > 2 * err:
            assert int(np.argmax(lg)) == O.greedy(lo), f"step {i}: greedy pick differs"
    g.close()
    o.close()
    return worst


# ---------------------------------------------------------------- fused GEMV forms
@pytest.mark.parametrize("dtype,in_dim,out_dim", [(12, 2048, 3072), (14, 8192, 2048), (2, 2048, 512),
                                                  (8, 4096, 1000), (14, 2048, 4096)])
@pytest.mark.parametrize("xmode", [0, 1, 2])
def test_fused_gemv_forms(torch_cuda, dtype, in_dim, out_dim, xmode):
    torch = torch_cuda
    from m3_avm_b200 import matvec_quant as MQ

    raw = synth.weights(dtype, in_dim, out_dim, seed=in_dim + out_dim + xmode)
    x = synth.activations(in_dim, 3) * np.float32(3.0)
    x2 = synth.activations(in_dim, 4)
    gamma = synth.activations(in_dim, 5)
    res = synth.activations(out_dim, 6) * np.float32(100.0)
    if xmode == 1:
        xin = O.rms_norm(x, gamma)
    elif xmode == 2:
        with np.errstate(over="ignore"):
            xin = (x * (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))) * x2).astype(np.float32)
    else:
        xin = x
    ref = O.matvec_quant(xin, raw, dtype, in_dim, out_dim)
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    for with_res in (False, True):
        y = MQ.matvec_fused_dev(T(x), T(raw), dtype, in_dim, out_dim, xmode=xmode, x2=T(x2),
                                gamma=T(gamma) if xmode == 1 else None, res=T(res) if with_res else None)
        torch.cuda.synchronize()
        got = y.cpu().numpy().astype(np.float64)
        want = ref.astype(np.float64) + (res if with_res else 0.0)
        bound = O.gemv_bound(raw, dtype, in_dim, out_dim, xin) + (np.abs(res) * 2.0 ** -23 if with_res else 0.0)
        bad = np.nonzero(np.abs(got - want) > bound + 1e-30)[0]
        assert bad.size == 0, (with_res, bad[:5], np.abs(got - want)[bad[:5]], bound[bad[:5]])


@pytest.mark.parametrize("dtype,in_dim,F", [(12, 2048, 8192), (8, 2048, 1000 // 8 * 8), (14, 2048, 512)])
def test_fused_gemv_swiglu_epilogue(torch_cuda, dtype, in_dim, F):
    torch = torch_cuda
    from m3_avm_b200 import matvec_quant as MQ

    gate = synth.weights(dtype, in_dim, F, seed=F + 1)
    up = synth.weights(dtype, in_dim, F, seed=F + 2)
    rb = gate.size // F
    inter = np.concatenate([gate.reshape(F // 8, 8 * rb), up.reshape(F // 8, 8 * rb)], axis=1).reshape(-1)
    x = synth.activations(in_dim, 9)
    gamma = synth.activations(in_dim, 10)
    xin = O.rms_norm(x, gamma)
    g = O.matvec_quant(xin, gate, dtype, in_dim, F).astype(np.float64)
    u = O.matvec_quant(xin, up, dtype, in_dim, F).astype(np.float64)
    with np.errstate(over="ignore"):
        want = g / (1.0 + np.exp(-g)) * u
    dev = torch.device("cuda:0")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    y = MQ.matvec_fused_dev(T(x), T(inter), dtype, in_dim, 2 * F, xmode=MQ.X_RMSNORM, gamma=T(gamma), swiglu=True)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    bg = O.gemv_bound(gate, dtype, in_dim, F, xin)
    bu = O.gemv_bound(up, dtype, in_dim, F, xin)
    with np.errstate(over="ignore"):
        sil = np.abs(g / (1.0 + np.exp(-g)))
    tol = 1.1 * bg * np.abs(u) + sil * bu + np.abs(want) * (np.abs(g) + 1.0) * 2.0 ** -20 + 1e-30
    bad = np.nonzero(np.abs(got - want) > tol)[0]
    assert bad.size == 0, (bad[:5], got[bad[:5]], want[bad[:5]], tol[bad[:5]])


def test_fused_gemv_rejects_shapes_without_tensor_core_plan(torch_cuda):
    torch = torch_cuda
    from m3_avm_b200 import _lib
    from m3_avm_b200 import matvec_quant as MQ

    raw = torch.zeros(210 * 4, dtype=torch.uint8, device="cuda:0")
    x = torch.zeros(1024, device="cuda:0")
    with pytest.raises(_lib.M3GError):  # Q6_K rows of 840 bytes are not 16-byte multiples
        MQ.matvec_fused_dev(x, raw, 14, 1024, 1)


# ---------------------------------------------------------------- whole steps
def test_decode_well_conditioned_teacher_forced(torch_cuda):
    T = model.synthetic_tensors(WELL, 11)
    toks = model.prompt_tokens(WELL, 24, 12)
    teacher_forced(WELL, T, toks)


def test_decode_head_dim_128_mixed_dtypes(torch_cuda):
    T = mixed_tensors(HD128, 13)
    toks = model.prompt_tokens(HD128, 12, 14)
    teacher_forced(HD128, T, toks)


def test_decode_llama_1b_shape_teacher_forced(torch_cuda):
    T = model.synthetic_tensors(model.LLAMA_1B, 1)
    toks = model.prompt_tokens(model.LLAMA_1B, 3, 2)
    teacher_forced(model.LLAMA_1B, T, toks, max_pos=8)


# ---------------------------------------------------------------- the device loop
def test_generate_equals_host_loop_and_graph_equals_eager(torch_cuda):
    T = model.synthetic_tensors(WELL, 21)
    prompt = model.prompt_tokens(WELL, 9, 22)
    n_gen = 12
    g = gpu_decoder(WELL, T, 64)
    toks = g.generate(prompt, n_gen)
    assert g.pos == len(prompt) + n_gen - 1
    assert np.array_equal(g.tokens(0, len(prompt)), prompt)
    assert np.array_equal(g.tokens(len(prompt), n_gen), toks)
    # the same loop driven from the host, eager launches
    h = gpu_decoder(WELL, T, 64)
    h.set_graph(False)
    for t in prompt[:-1]:
        h.forward_one(int(t))
    logits = h.forward_one(int(prompt[-1]))
    seq = []
    for i in range(n_gen):
        nxt = h.sample(logits)
        seq.append(nxt)
        if i + 1 < n_gen:
            logits = h.forward_one(nxt)
    assert np.array_equal(np.array(seq, np.uint32), toks)
    # graph and eager steps agree bit for bit
    g.truncate_kv_cache(len(prompt) - 1)
    a = g.forward_one(int(prompt[-1]))
    h.truncate_kv_cache(len(prompt) - 1)
    b = h.forward_one(int(prompt[-1]))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    g.close()
    h.close()


def test_truncate_replays_bit_for_bit(torch_cuda):
    T = model.synthetic_tensors(WELL, 31)
    g = gpu_decoder(WELL, T, 16)
    a = [g.forward_one(t) for t in (5, 17, 99)]
    g.truncate_kv_cache(1)
    b = [g.forward_one(t) for t in (17, 99)]
    for x, y in zip(a[1:], b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    g.clear_kv_cache()
    assert np.array_equal(g.forward_one(5).view(np.uint32), a[0].view(np.uint32))
    g.close()


def test_decoder_failure_rules(torch_cuda):
    from m3_avm_b200 import _lib
    from m3_avm_b200.decoder import GpuDecoder

    T = model.synthetic_tensors(WELL, 41)
    d = GpuDecoder(WELL, max_pos=2)
    with pytest.raises(_lib.M3GError):  # tensors missing
        d.forward_one(0)
    d.upload_all(T)
    with pytest.raises(_lib.M3GError):  # token outside the vocabulary
        d.forward_one(WELL.vocab)
    with pytest.raises(_lib.M3GError):  # nothing to continue from
        d.generate([], 2)
    with pytest.raises(_lib.M3GError):  # a norm must be f32
        d.upload(model.SLOT_OUT_NORM, np.ones(WELL.hidden, np.float32), 1)
    with pytest.raises(_lib.M3GError):  # short bytes
        d.upload(model.SLOT_OUT, T[model.SLOT_OUT][0][:100], 14)
    d.forward_one(1)
    d.forward_one(2)
    with pytest.raises(_lib.M3GError):  # KV cache full
        d.forward_one(3)
    with pytest.raises(_lib.M3GError):
        GpuDecoder(model.LlamaShape(n_heads=24))  # head_dim 2048 / 24 is not whole
    d.close()


def test_decoder_from_gguf_file_equals_direct_upload(torch_cuda, tmp_path):
    from m3_avm_b200 import gguf as G

    p = str(tmp_path / "well.gguf")
    G.write_synthetic_model(p, WELL, seed=51)
    dec, shape = G.load_decoder(p, max_pos=16)
    assert shape == WELL
    direct = gpu_decoder(WELL, model.synthetic_tensors(WELL, 51), 16)
    for t in (3, 999, 4095):
        a = dec.forward_one(t)
        b = direct.forward_one(t)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    dec.close()
    direct.close()
