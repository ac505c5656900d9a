"""Sharded decode (one process per GPU, NCCL) against the single-GPU engine.

Each rank keeps its rows of ffn_gate/up/down and the vocab head (or only of
the head, every rank keeping the layers); every row is computed exactly as on
one GPU, so the sharded steps must reproduce the single-GPU logits and greedy
tokens bit for bit -- with the rows exchanged by peer stores from the GEMV
epilogues, with NCCL all-gathers, and with the head split alone (greedy keys
merged by an NCCL all-reduce, or by peer atomics into per-step-parity slots
with no collective per step, across a cache truncation).  Also: a rank that never
joins makes creation give up with M3G_ETIMEOUT (host-side failure detection,
nothing waits on the GPU).
"""
import os

import numpy as np
import pytest

from m3_avm_b200 import model

pytestmark = pytest.mark.gpu

SHAPE = model.LlamaShape(n_layers=2, hidden=2048, ffn=2048, n_heads=32, n_kv_heads=8, vocab=4099,
                         rope_theta=500000.0, embd_dtype=12, attn_dtype=2, gate_up_dtype=8, down_dtype=14,
                         head_dtype=14)
PROMPT = [5, 77, 1000, 4098, 3]
N_GEN = 6


def _run(shape, rank, world, uid, p2p=1, shard_ffn=1):
    from m3_avm_b200 import matvec_quant as MQ
    from m3_avm_b200.decoder import GpuDecoder

    MQ.set_tuning("decode_p2p", p2p)
    MQ.set_tuning("decode_shard_ffn", shard_ffn)

    d = GpuDecoder(shape, max_pos=32, device=rank, rank=rank, world=world, nccl_id=uid, timeout_s=60)
    d.upload_all(model.synthetic_tensors(shape, 3))
    logits = [d.forward_one(t) for t in PROMPT]
    d.clear_kv_cache()
    toks = d.generate(PROMPT, N_GEN)
    exchange = d.exchange
    d.close()
    return [lg.tobytes() for lg in logits], toks.tobytes(), exchange


def _rank(rank, world, uid, p2p, shard_ffn, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    torch.cuda.set_device(rank)
    try:
        q.put((rank, _run(SHAPE, rank, world, uid, p2p, shard_ffn)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))


@pytest.mark.parametrize("p2p,shard_ffn,exchange", [(1, 1, "peer-stores"), (0, 1, "nccl"), (0, 0, "head-only"),
                                                    (1, 0, "head-only-peer")],
                         ids=["peer-stores", "nccl", "head-only", "head-only-peer"])
def test_sharded_decode_matches_single_gpu_bitwise(p2p, shard_ffn, exchange):
    import multiprocessing as mp

    import torch

    from m3_avm_b200 import sharded

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    uid = sharded.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, p2p, shard_ffn, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
    want_logits, want_toks, single = _run(SHAPE, 0, 1, None)
    assert single == "single"
    for r in range(world):
        got_logits, got_toks, got_exchange = res[r]
        assert got_exchange == exchange
        assert got_toks == want_toks
        for a, b in zip(got_logits, want_logits):
            assert a == b


def _lonely(uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from m3_avm_b200 import _lib
    from m3_avm_b200.decoder import GpuDecoder

    try:
        GpuDecoder(SHAPE, max_pos=8, device=0, rank=0, world=2, nccl_id=uid, timeout_s=3.0)
        q.put(("joined", 0))
    except _lib.M3GError as e:
        q.put(("error", e.code))


def test_sharded_decoder_rank_that_never_joins_times_out():
    import multiprocessing as mp

    from m3_avm_b200 import _lib, sharded

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(sharded.unique_id(), q))
    p.start()
    p.join(120)
    assert p.exitcode == 0
    assert q.get(timeout=5) == ("error", _lib.M3G_ETIMEOUT)
