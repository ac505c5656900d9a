"""GGUF ingest on the CPU: the reader and writer against each other and against
the independent `gguf` Python package (GGUFReader / GGUFWriter), the model
keys of ModelConfig::from_gguf, and the tied-head fallback."""
import os

import numpy as np
import pytest

from m3_avm_b200 import gguf as G
from m3_avm_b200 import model

SMALL = model.LlamaShape(n_layers=2, hidden=256, ffn=512, n_heads=4, n_kv_heads=2, vocab=300, rope_theta=123456.0,
                         embd_dtype=12, attn_dtype=2, gate_up_dtype=8, down_dtype=14, head_dtype=14)


def test_synthetic_model_roundtrip(tmp_path):
    p = str(tmp_path / "m.gguf")
    G.write_synthetic_model(p, SMALL, seed=5)
    g = G.read_gguf(p)
    assert g.version == 3 and g.data_offset % 32 == 0
    assert G.shape_from_gguf(g) == SMALL
    want = model.synthetic_tensors(SMALL, 5)
    got = G.tensors_from_gguf(g, SMALL)
    assert set(got) == set(want)
    for slot, (arr, dt) in want.items():
        assert got[slot][1] == dt
        assert np.array_equal(np.asarray(got[slot][0]), np.ascontiguousarray(arr).view(np.uint8).reshape(-1))


def test_independent_reader_reads_our_file(tmp_path):
    gg = pytest.importorskip("gguf")
    p = str(tmp_path / "m.gguf")
    G.write_synthetic_model(p, SMALL, seed=6)
    r = gg.GGUFReader(p)
    ours = G.read_gguf(p)
    assert len(r.tensors) == len(ours.tensors)
    for t in r.tensors:
        mine = ours.find(t.name)
        assert mine is not None and int(t.tensor_type) == mine.dtype
        assert [int(d) for d in t.shape] == mine.dims
        assert np.array_equal(np.asarray(t.data).view(np.uint8).reshape(-1), np.asarray(ours.tensor_bytes(t.name)))
    f = r.fields["llama.embedding_length"]
    assert int(f.parts[f.data[0]][0]) == SMALL.hidden


def test_our_reader_reads_independent_writer(tmp_path):
    gg = pytest.importorskip("gguf")
    from m3_avm_b200 import synth

    p = str(tmp_path / "w.gguf")
    w = gg.GGUFWriter(p, "llama")
    w.add_block_count(1)
    w.add_embedding_length(256)
    w.add_feed_forward_length(512)
    w.add_head_count(4)
    w.add_head_count_kv(4)
    w.add_rope_freq_base(500000.0)
    w.add_token_list([f"t{i}" for i in range(77)])
    q4k = synth.weights(12, 256, 64, seed=1)
    f32 = np.arange(256, dtype=np.float32)
    w.add_tensor("blk.0.ffn_gate.weight", q4k, raw_shape=(64, 144), raw_dtype=gg.GGMLQuantizationType.Q4_K)
    w.add_tensor("output_norm.weight", f32)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = G.read_gguf(p)
    t = g.find("blk.0.ffn_gate.weight")
    assert t.dtype == 12 and t.dims == [256, 64]
    assert np.array_equal(np.asarray(g.tensor_bytes("blk.0.ffn_gate.weight")), q4k)
    assert np.array_equal(np.asarray(g.tensor_bytes("output_norm.weight")).view(np.float32), f32)
    s = G.shape_from_gguf(g)
    assert (s.n_layers, s.hidden, s.ffn, s.n_heads, s.vocab, s.rope_theta) == (1, 256, 512, 4, 77, 500000.0)


def test_tied_head_falls_back_to_token_embd(tmp_path):
    tens = model.synthetic_tensors(SMALL, 7)
    names = G.slot_names(SMALL)
    entries = []
    for slot in sorted(tens):
        if slot == model.SLOT_OUT:
            continue
        arr, dt = tens[slot]
        m = SMALL.matrix(slot)
        entries.append((names[slot], [SMALL.hidden] if m is None else [m[1], m[2]], dt, arr))
    p = str(tmp_path / "tied.gguf")
    G.write_gguf(p, {"llama.embedding_length": SMALL.hidden, "llama.block_count": SMALL.n_layers,
                     "llama.feed_forward_length": SMALL.ffn, "llama.attention.head_count": SMALL.n_heads,
                     "llama.attention.head_count_kv": SMALL.n_kv_heads, "llama.vocab_size": SMALL.vocab}, entries)
    g = G.read_gguf(p)
    s = G.shape_from_gguf(g)
    got = G.tensors_from_gguf(g, s)
    assert np.array_equal(np.asarray(got[model.SLOT_OUT][0]), np.asarray(got[model.SLOT_EMBD][0]))


def test_rejects_bad_magic(tmp_path):
    p = str(tmp_path / "bad.gguf")
    with open(p, "wb") as f:
        f.write(b"XXXX" + bytes(40))
    with pytest.raises(ValueError):
        G.read_gguf(p)
    with open(p, "wb") as f:
        f.write(b"GGUF" + bytes(6))
    with pytest.raises(ValueError):
        G.read_gguf(p)
    os.remove(p)
