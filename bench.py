#!/usr/bin/env python
"""Benchmark of the fused Q4_K GEMV (and the CPU reference beside it).

Workload (the headline metric): one Q4_K GEMV of 14336 output rows over 4096
inputs (the Llama-3-8B FFN gate/up shape), fp32 x ~ N(0, 1), seeded synthetic
GGUF weights.  A step is one GEMV.  The weights rotate over enough resident
copies that the set is larger than three times the L2, so every step streams
its 33 MB from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` is whole-job HBM GB/s of algorithmic
bytes (weights + x + y) with inputs resident; `e2e` is the same metric through
the GpuOffload-shaped C ABI call with host x and y (copies in the timed
region).  Under torchrun every rank runs its own GEMV stream (weak scaling, no
data-path collective); the time is the max over ranks.

The second half of the metric, decode tokens/s, is the `decode` object of the
same line: greedy decode of a Llama-3.2-1B-shaped model (Q4_K_M mix) through
the device-resident engine, 128 prompt tokens then 256 generated, with the
C restatement of the reference's CPU forward pass timed beside it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

IN_DIM, OUT_DIM, DTYPE = 4096, 14336, 12
WORKLOAD = "q4k_gemv_14336x4096"
METRIC = "Q4_K GEMV HBM GB/s (% of peak) @4096x14336; 1B decode tokens/sec"


def algorithmic_bytes(in_dim: int, out_dim: int, dtype: int, batch: int = 1) -> int:
    """Weight bytes + 4*B*in + 4*B*out (each weight byte, x and y touched once)."""
    be, bb = {12: (256, 144), 14: (256, 210), 8: (32, 34), 2: (32, 18)}[dtype]
    return in_dim * out_dim // be * bb + 4 * batch * in_dim + 4 * batch * out_dim


def measured_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def committed_traffic(kernel: str, workload: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(f"{kernel}@{workload}")
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def cpu_gemv_rate(threads: int, target_s: float, max_calls: int | None = None) -> dict:
    """The oracle's port of the reference AVX2 matvec_q4k on this host's cores (CPU baseline)."""
    from oracle import oracle as O
    from m3_avm_b200 import synth

    raw = synth.weights(DTYPE, IN_DIM, OUT_DIM, seed=1)
    x = synth.activations(IN_DIM, seed=2)
    O.matvec_quant(x, raw, DTYPE, IN_DIM, OUT_DIM, threads=threads)  # warm
    times = []
    t_end = time.perf_counter() + target_s
    while time.perf_counter() < t_end and (max_calls is None or len(times) < max_calls):
        t0 = time.perf_counter()
        O.matvec_quant(x, raw, DTYPE, IN_DIM, OUT_DIM, threads=threads)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    gbs = algorithmic_bytes(IN_DIM, OUT_DIM, DTYPE) / med / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} full {OUT_DIM}x{IN_DIM} Q4_K GEMVs (C restatement of the reference AVX2 "
                      f"matvec_q4k, {threads} OpenMP threads), median {med * 1e3:.3f} ms",
            "median_s": med}


DECODE_PROMPT, DECODE_GEN = 128, 256


def _decode_run(args, dev, world, shape, tensors, prompt) -> dict:
    """One decoder: warm-up, then device-timed generation and the e2e call."""
    import torch
    import torch.distributed as dist

    from m3_avm_b200.decoder import GpuDecoder

    max_pos = DECODE_PROMPT + DECODE_GEN + 8
    if world > 1:
        dec = GpuDecoder.from_torch_dist(shape, max_pos=max_pos, device=dev.index or 0, timeout_s=120)
    else:
        dec = GpuDecoder(shape, max_pos=max_pos, device=dev.index or 0)
    dec.upload_all(tensors)
    exchange = dec.exchange
    dec.set_graph(not args.no_graph)
    st = torch.cuda.ExternalStream(dec.stream, device=dev)
    # warm-up: one full prompt + a few steps (graph capture, lazy setup)
    dec.prefill_logits(prompt)
    dec.run_async(8)
    dec.sync()
    dec.clear_kv_cache()
    dec.prefill_logits(prompt)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    dec.run_async(DECODE_GEN - 1)  # the first generated token is the prefill's pick
    e1.record(st)
    dec.sync()
    gen_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([gen_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gen_ms = float(t.item())
    toks = dec.tokens(DECODE_PROMPT, DECODE_GEN)
    # e2e: the public call a user makes, host prompt in, host tokens out
    dec.clear_kv_cache()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    toks2 = dec.generate(prompt, DECODE_GEN)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    dec.close()
    return {"gen_ms": gen_ms, "tok_s": (DECODE_GEN - 1) / (gen_ms / 1e3), "e2e_s": e2e_s, "exchange": exchange,
            "toks": toks, "match": bool((toks == toks2).all())}


def decode_leg(args, dev, world: int = 1) -> dict:
    """Greedy decode of the Llama-3.2-1B-shaped model (16 layers, hidden 2048,
    FFN 8192, 32/8 heads x 64, vocab 128256, Q4_K attention/gate/up/embedding,
    Q6_K down and head), seeded synthetic weights: a 128-token prompt, then
    256 generated tokens, all steps device-resident.  Under torchrun the engine
    is row-sharded over the ranks in two ways, both measured: the vocab head
    alone (every rank keeps the layers; the greedy keys merge by peer atomics
    over NVLink, or by one NCCL all-reduce per token where peers cannot be
    mapped) and the FFN plus the head (rows exchanged every layer); the time is
    the max over ranks (strong scaling: one model, one sequence)."""
    from m3_avm_b200 import matvec_quant as MQ
    from m3_avm_b200 import model

    shape = model.LLAMA_1B
    tensors = model.synthetic_tensors(shape, seed=1)
    prompt = model.prompt_tokens(shape, DECODE_PROMPT, seed=2)
    modes = {}
    if world > 1:
        for name, shard_ffn in (("head-only", 0), ("ffn+head", 1)):
            MQ.set_tuning("decode_shard_ffn", shard_ffn)
            modes[name] = _decode_run(args, dev, world, shape, tensors, prompt)
        MQ.set_tuning("decode_shard_ffn", 1)
        best = max(modes, key=lambda k: modes[k]["tok_s"])
        r = modes[best]
    else:
        r = _decode_run(args, dev, world, shape, tensors, prompt)
    tok_s, gen_ms, e2e_s = r["tok_s"], r["gen_ms"], r["e2e_s"]
    bytes_tok = shape.weight_bytes_per_token()
    peaks, kind = measured_peaks()
    peak = float(peaks["hbm_gbs"])
    nccl_per_token = {"nccl": 2 * shape.n_layers + 1, "peer-stores": 0, "head-only": 1, "head-only-peer": 0,
                      "single": 0}
    out = {
        "workload": "llama-3.2-1b-shaped greedy decode, Q4_K_M mix (Q4_K attn/gate/up/embd, Q6_K down/head)",
        "prompt_tokens": DECODE_PROMPT, "generated_tokens": DECODE_GEN,
        "tokens_per_s": round(tok_s, 1), "us_per_token": round(gen_ms * 1e3 / (DECODE_GEN - 1), 2),
        "timing": "CUDA events on the decoder stream around the 255 generation steps after the prompt",
        "roofline": {"bound": "hbm", "weight_bytes_per_token": bytes_tok,
                     "achieved_gbs": round(bytes_tok * tok_s / 1e9, 1), "peak": peak, "peak_kind": kind,
                     "frac": round(bytes_tok * tok_s / 1e9 / peak, 4),
                     "roofline_tokens_per_s": round(peak * 1e9 / bytes_tok, 1)},
        "e2e": {"value": round(DECODE_GEN / e2e_s, 1), "unit": "tokens/s",
                "api": "m3g_decoder_prefill + m3g_decoder_generate (host prompt in, host tokens out; "
                       "includes the 128-token prefill)",
                "h2d_bytes_per_step": 4 * DECODE_PROMPT, "d2h_bytes_per_step": 4 * DECODE_GEN,
                "seconds": round(e2e_s, 4)},
        "tokens_match_e2e": r["match"],
        "graph": not args.no_graph,
        "gpu_launches_per_token": 1 + 5 * shape.n_layers + 2,
        "n_gpus": world,
        "parallelism": f"rows{world} ({r['exchange']})" if world > 1 else "single GPU",
        "scaling": "strong",
    }
    if world > 1:
        out["nccl_collectives_per_token"] = nccl_per_token.get(r["exchange"])
        out["roofline"]["note"] = "weight bytes of the whole model per token; each GPU streams its share"
        out["modes"] = {k: {"tokens_per_s": round(v["tok_s"], 1), "exchange": v["exchange"],
                            "e2e_tokens_per_s": round(DECODE_GEN / v["e2e_s"], 1)} for k, v in modes.items()}
        out["modes_tokens_match"] = bool(all((v["toks"] == r["toks"]).all() for v in modes.values()))
    if not args.no_cpu and world == 1:
        out["cpu_baseline"] = cpu_decode_rate(shape, tensors, prompt)
    return out


BATCHED_IN, BATCHED_OUT, BATCHED_B = 8192, 28672, (1, 4, 16, 32, 64)


def batched_leg(args, dev, rank: int = 0, world: int = 1) -> dict:
    """Batched decode GEMM: Q4_K 28672 x 8192 weights against X of B x 8192,
    B in {1, 4, 16, 32, 64}; the output rows are split evenly over the ranks
    (each GPU holds its row shard, no collective); rotating resident weight
    copies (> 3x L2), CUDA events around CUDA-graph replays, the time taken as
    the max over ranks between barriers.  Effective GB/s counts the whole
    weight once plus X and Y (4*B*in + 4*B*out); TFLOP/s counts 2*B*in*out."""
    import torch
    import torch.distributed as dist

    from m3_avm_b200 import _lib, synth
    from m3_avm_b200.inference_gpu import GpuOffload

    raw = synth.weights(DTYPE, BATCHED_IN, BATCHED_OUT, seed=5)
    rows = BATCHED_OUT // world
    rb = raw.size // BATCHED_OUT
    shard = raw[rank * rows * rb:(rank + 1) * rows * rb]
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    n_copies = max(2, math.ceil(3 * l2 / shard.size))
    g = GpuOffload.try_new(BATCHED_IN, rows, device=dev.index or 0)
    for c in range(n_copies):
        if not g.upload(c, DTYPE, shard, BATCHED_IN, rows):
            raise RuntimeError("upload failed: " + _lib.last_error())
    out = {"workload": f"q4k_batched_{BATCHED_OUT}x{BATCHED_IN}", "weight_copies": n_copies, "sweep": {},
           "parallelism": f"rows{world}" if world > 1 else "single GPU", "rows_per_gpu": rows}
    peaks, kind = measured_peaks()
    for B in BATCHED_B:
        X = torch.from_numpy(synth.activations(BATCHED_IN, seed=6, batch=B)).to(dev)
        Y = torch.empty((B, rows), dtype=torch.float32, device=dev)
        cap = torch.cuda.Stream(dev)
        reps = max(3, min(60, int(2000 / B)))
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cap, capture_error_mode="thread_local"):
            for c in range(n_copies):
                g.matvec_dev(c, X, Y, stream=cap.cuda_stream)
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        us = float(ms.item()) * 1e3 / (reps * n_copies)
        abytes = algorithmic_bytes(BATCHED_IN, BATCHED_OUT, DTYPE, batch=B)
        flops = 2.0 * B * BATCHED_IN * BATCHED_OUT
        out["sweep"][str(B)] = {"us": round(us, 2), "gbs": round(abytes / us / 1e3, 1),
                                "tflops": round(flops / us / 1e6, 2),
                                "frac_of_hbm": round(abytes / us / 1e3 / float(peaks["hbm_gbs"]) / world, 4)}
        del gr
    g.close()
    out["kernel"] = ("k_umma_xprep + k_umma_q4k (tcgen05, up to 64 columns per pass, "
                     "fp16 sc*q operand in TMEM); B=1 takes k_gemv_mma")
    out["frac_of_hbm"] = "of the measured peak of all the GPUs used"
    return out


def cpu_decode_rate(shape, tensors, prompt, n_tokens: int = 3) -> dict:
    """The oracle's restatement of forward_one (reference CPU path) on the host cores."""
    from oracle import oracle as O

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    dec = O.Decoder(shape.n_layers, shape.hidden, shape.ffn, shape.n_heads, shape.n_kv_heads, shape.vocab,
                    shape.rope_theta, 64, tensors, threads=threads)
    t0 = time.perf_counter()
    dec.forward(int(prompt[0]))  # dequantises and caches the f32 head, like the reference's first token
    first = time.perf_counter() - t0
    times = []
    for t in prompt[1:1 + n_tokens]:
        t0 = time.perf_counter()
        dec.forward(int(t))
        times.append(time.perf_counter() - t0)
    dec.close()
    med = statistics.median(times)
    return {"value": round(1.0 / med, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n_tokens} forward_one steps after a first step of {first:.2f} s (C restatement of "
                      f"RealInference::forward_one with matvec_quant and the f32-cached head, {threads} OpenMP "
                      f"threads), median {med * 1e3:.1f} ms"}


def run_reference(args) -> int:
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O
    from m3_avm_b200 import synth

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    raw = synth.weights(DTYPE, IN_DIM, OUT_DIM, seed=1)
    x = synth.activations(IN_DIM, seed=2)
    # one step = one full GEMV on the host cores, unless K of them would not fit
    # in ~2 minutes; then a step is a contiguous slice of rows of that GEMV.
    t0 = time.perf_counter()
    O.matvec_quant(x, raw, DTYPE, IN_DIM, OUT_DIM, threads=threads)
    one = time.perf_counter() - t0
    rows = OUT_DIM
    budget = 120.0
    if one * (args.steps + args.warmup) > budget:
        rows = max(8, int(OUT_DIM * budget / (one * (args.steps + args.warmup))))
    row_bytes = IN_DIM // 256 * 144
    sub = raw[: rows * row_bytes]
    for _ in range(args.warmup):
        O.matvec_quant(x, sub, DTYPE, IN_DIM, rows, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.matvec_quant(x, sub, DTYPE, IN_DIM, rows, threads=threads)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    gbs = algorithmic_bytes(IN_DIM, rows, DTYPE) / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows_per_step": rows, "in_dim": IN_DIM, "dtype": "Q4_K"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {OUT_DIM} rows x {IN_DIM} Q4_K per step (C restatement of the "
                                   f"reference AVX2 matvec_q4k; the Rust crate cannot be built here)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_decode:
        from m3_avm_b200 import model

        shape = model.LLAMA_1B
        line["decode"] = {"cpu_baseline": cpu_decode_rate(shape, model.synthetic_tensors(shape, seed=1),
                                                          model.prompt_tokens(shape, DECODE_PROMPT, seed=2))}
        line["decode"]["tokens_per_s"] = line["decode"]["cpu_baseline"]["value"]
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from m3_avm_b200 import _lib, synth
    from m3_avm_b200.inference_gpu import GpuOffload

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    lib = _lib.load()
    dev = torch.device("cuda", local)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024

    raw = synth.weights(DTYPE, IN_DIM, OUT_DIM, seed=1 + rank)
    wbytes = raw.size
    n_copies = max(2, math.ceil(3 * l2 / wbytes))
    g = GpuOffload.try_new(IN_DIM, OUT_DIM, device=local)
    if g is None:
        raise RuntimeError("GpuOffload.try_new failed: " + _lib.last_error())
    for c in range(n_copies):
        if not g.upload(c, DTYPE, raw, IN_DIM, OUT_DIM):
            raise RuntimeError("upload failed: " + _lib.last_error())
    x = torch.from_numpy(synth.activations(IN_DIM, seed=2)).to(dev)
    y = torch.empty(OUT_DIM, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i, st):
        g.matvec_dev(i % n_copies, x, y, stream=st.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # The timed steps replay CUDA graphs that hold one launch per weight copy,
    # so the host's launch cost does not gate the GPU.
    cap = torch.cuda.Stream(dev)
    graphs = []
    if not args.no_graph:
        for n_launch in sorted({n_copies, args.steps % n_copies} - {0}, reverse=True):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=cap, capture_error_mode="thread_local"):
                for c in range(n_launch):
                    step(c, cap)
            graphs.append((n_launch, gr))
    gmap = dict(graphs)

    def run_steps(k, marks=None):
        if args.no_graph:
            for i in range(k):
                step(i, stream)
            return
        full, rest = divmod(k, n_copies)
        # Window boundaries for the median and best window (at most ~64 event
        # records in the timed region, so they do not slow the replays).
        per_win = max(1, full // 64)
        for r in range(full):
            gmap[n_copies].replay()
            if marks is not None and (r + 1) % per_win == 0:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(stream)
                marks.append((ev, per_win * n_copies))
        if rest:
            if rest not in gmap:
                for i in range(rest):
                    step(i, stream)
            else:
                gmap[rest].replay()

    run_steps(args.warmup)
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.25)
    barrier()
    launches0 = int(lib.m3g_launch_count())
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    marks = [(ev0, 0)]
    run_steps(args.steps, marks)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    host_launches = int(lib.m3g_launch_count()) - launches0
    win_us = [a.elapsed_time(b) * 1e3 / n for (a, _), (b, n) in zip(marks, marks[1:])]
    windows = ({"median_us": round(statistics.median(win_us), 3), "best_us": round(min(win_us), 3),
                "windows": len(win_us), "steps_per_window": marks[1][1]} if win_us else None)
    launches = args.steps if not args.no_graph else host_launches
    ms = ev0.elapsed_time(ev1)
    barrier()
    clocks = sampler.stop()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    per_step_s = ms_max / 1e3 / args.steps
    abytes = algorithmic_bytes(IN_DIM, OUT_DIM, DTYPE)
    value = abytes * world / per_step_s / 1e9

    # e2e: host x -> device, GEMV, device y -> host, through the C ABI offload call.
    xh = synth.activations(IN_DIM, seed=2)
    e2e_steps = 0 if args.no_e2e else min(args.steps, 5000)
    for i in range(min(args.warmup, 50)):
        g.matvec(i % n_copies, xh, IN_DIM, OUT_DIM)
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        if g.matvec(i % n_copies, xh, IN_DIM, OUT_DIM) is None:
            raise RuntimeError("offload matvec failed: " + _lib.last_error())
    e2e_s = (time.perf_counter() - t0) / max(e2e_steps, 1)
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = abytes * world / float(te.item()) / 1e9

    status = ctypes_status(lib, local)
    peaks, kind = measured_peaks()
    peak = float(peaks["hbm_gbs"])
    achieved = abytes / per_step_s / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": kind,
                "traffic": committed_traffic("k_gemv_mma", WORKLOAD), "kernel": "k_gemv_mma<MmaQ4K>",
                "algorithmic_bytes_per_launch": abytes}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        cpu = cpu_gemv_rate(threads, target_s=args.cpu_seconds)
        cpu.pop("median_s", None)

    decode = None
    if not args.no_decode:
        decode = decode_leg(args, dev, world)
    batched = None
    if not args.no_batched:
        batched = batched_leg(args, dev, rank, world)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "dtype": "Q4_K", "in_dim": IN_DIM, "out_dim": OUT_DIM,
                       "weight_copies": n_copies, "weight_set_mb": round(n_copies * wbytes / 2**20, 1),
                       "l2_mb": round(l2 / 2**20, 1), "l2": "inputs larger than L2 (rotating weight copies)",
                       "parallelism": f"replicas{world}"},
            "pct_of_measured_hbm_peak": round(100 * achieved / peak, 2),
            "pct_of_8tbps_spec": round(100 * achieved / 8000.0, 2),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "h2d_bytes_per_step": 4 * IN_DIM,
                    "d2h_bytes_per_step": 4 * OUT_DIM, "us_per_call": round(float(te.item()) * 1e6, 2),
                    "api": "m3g_offload_matvec (host x/y, resident weights)"},
            "gpu_launches": launches,
            "per_step_windows": windows,
            "timing": "CUDA events around CUDA-graph replays of the GEMV launches" if not args.no_graph
                      else "CUDA events around host-launched GEMVs",
            "clocks": clocks,
            "device_status": status,
            "decode": decode,
            "batched": batched,
        }
        print(json.dumps(line), flush=True)
    g.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_lmhead(args) -> int:
    """Vocab-head GEMV, Q6_K 128256 x 4096, rows sharded over the ranks plus one
    NCCL all-gather of the fp32 logits (strong scaling: total work fixed)."""
    import datetime

    import torch
    import torch.distributed as dist

    from m3_avm_b200 import _lib, sharded, synth

    in_dim, out_dim, dtype = 4096, 128256, 14
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        s = sharded.ShardedOffload.from_torch_dist(local, in_dim, out_dim, timeout_s=120)
    else:
        s = sharded.ShardedOffload(local, 0, 1, sharded.unique_id(), in_dim, out_dim, timeout_s=120)
    lib = _lib.load()
    raw = synth.weights(dtype, in_dim, out_dim, seed=1)
    _, rows_local, rpr, _, bytes_local = sharded.shard_plan(dtype, in_dim, out_dim, world, rank)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    n_copies = max(2, math.ceil(3 * l2 / max(bytes_local, 1)))
    for c in range(n_copies):
        if not s.upload(c, dtype, raw, in_dim, out_dim):
            raise RuntimeError("shard upload failed: " + _lib.last_error())
    x = torch.from_numpy(synth.activations(in_dim, seed=2)).to(dev)
    y = torch.zeros(s.gather_len(0), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def replay():  # one pass over the weight copies, launched from the host
        for c in range(n_copies):
            s.matvec_dev(c, x, y, stream=stream.cuda_stream)

    reps_w = max(1, args.warmup // n_copies)
    reps = max(1, args.steps // n_copies)
    for _ in range(reps_w):
        replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.25)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(reps):
        replay()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    steps = reps * n_copies
    t = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    per_step = float(t.item()) / 1e3 / steps
    ab = algorithmic_bytes(in_dim, out_dim, dtype)
    peaks, kind = measured_peaks()
    if rank == 0:
        line = {
            "metric": "Q6_K vocab-head GEMV + all-gather, effective GB/s @128256x4096", "value": round(ab / per_step / 1e9, 2),
            "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": reps_w * n_copies,
            "ms_per_step": round(per_step * 1e3, 6), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "q6k_lmhead_128256x4096_sharded", "rows_per_rank": rpr, "weight_copies": n_copies,
                       "parallelism": f"rows{world}+allgather", "l2": "inputs larger than L2 (rotating weight copies)"},
            "per_gpu_hbm_gbs": round(bytes_local / per_step / 1e9, 2),
            "pct_of_measured_hbm_peak_per_gpu": round(100 * bytes_local / per_step / 1e9 / float(peaks["hbm_gbs"]), 2),
            "clocks": clocks,
            "timing": "CUDA events around host-launched steps (GEMV + NCCL all-gather each), max over ranks",
        }
        print(json.dumps(line), flush=True)
    s.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_decode(args) -> int:
    """Decode only: the 1B-shaped greedy decode, `--steps` generated tokens
    after a 128-token prompt and `--warmup` untimed steps, on 1 GPU or row-
    sharded under torchrun.  value = tokens/s (device time, max over ranks)."""
    import datetime

    import torch
    import torch.distributed as dist

    from m3_avm_b200 import model
    from m3_avm_b200.decoder import GpuDecoder

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    shape = model.LLAMA_1B
    prompt = model.prompt_tokens(shape, DECODE_PROMPT, seed=2)
    steps = max(1, min(args.steps, 2048))
    max_pos = DECODE_PROMPT + args.warmup + steps + 8
    if world > 1:
        from m3_avm_b200 import matvec_quant as MQ

        MQ.set_tuning("decode_shard_ffn", 0 if args.decode_mode == "head-only" else 1)
        dec = GpuDecoder.from_torch_dist(shape, max_pos=max_pos, device=local, timeout_s=120)
    else:
        dec = GpuDecoder(shape, max_pos=max_pos, device=local)
    dec.upload_all(model.synthetic_tensors(shape, seed=1))
    dec.set_graph(not args.no_graph)
    st = torch.cuda.ExternalStream(dec.stream, device=dev)
    dec.prefill_logits(prompt)
    dec.run_async(args.warmup)
    dec.sync()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    dec.run_async(steps)
    e1.record(st)
    dec.sync()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    exchange = dec.exchange
    dec.close()
    peaks, kind = measured_peaks()
    bytes_tok = shape.weight_bytes_per_token()
    tok_s = steps / (ms / 1e3)
    if rank == 0:
        print(json.dumps({
            "metric": "1B decode tokens/sec", "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "llama-3.2-1b-shaped greedy decode, Q4_K_M mix", "prompt_tokens": DECODE_PROMPT,
                       "parallelism": f"rows{world} ({exchange})" if world > 1 else "single GPU",
                       "graph": not args.no_graph},
            "roofline": {"bound": "hbm", "weight_bytes_per_token": bytes_tok,
                         "achieved": round(bytes_tok * tok_s / 1e9, 1), "peak": float(peaks["hbm_gbs"]),
                         "unit": "GB/s", "frac": round(bytes_tok * tok_s / 1e9 / float(peaks["hbm_gbs"]), 4),
                         "peak_kind": kind},
            "gpu_launches": steps * (1 + 5 * shape.n_layers + 2),
            "clocks": clocks,
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_batched(args) -> int:
    """One batched Q4_K 28672 x 8192 GEMM with X of --batch columns, `--steps`
    timed launches over rotating weight copies (a small case for profiling)."""
    import torch

    from m3_avm_b200 import synth
    from m3_avm_b200.inference_gpu import GpuOffload

    dev = torch.device("cuda", 0)
    B = args.batch
    raw = synth.weights(DTYPE, BATCHED_IN, BATCHED_OUT, seed=5)
    n_copies = 2
    g = GpuOffload.try_new(BATCHED_IN, BATCHED_OUT, device=0)
    for c in range(n_copies):
        g.upload(c, DTYPE, raw, BATCHED_IN, BATCHED_OUT)
    X = torch.from_numpy(synth.activations(BATCHED_IN, seed=6, batch=B)).to(dev)
    Y = torch.empty((B, BATCHED_OUT), dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        g.matvec_dev(i % n_copies, X, Y, stream=st.cuda_stream)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        g.matvec_dev(i % n_copies, X, Y, stream=st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    g.close()
    abytes = algorithmic_bytes(BATCHED_IN, BATCHED_OUT, DTYPE, batch=B)
    print(json.dumps({"metric": f"Q4_K batched GEMM effective GB/s @{BATCHED_OUT}x{BATCHED_IN}, B={B}",
                      "value": round(abytes / us / 1e3, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5), "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                      "config": {"workload": f"q4k_batched_{BATCHED_OUT}x{BATCHED_IN}", "batch": B,
                                 "weight_copies": n_copies},
                      "tflops": round(2.0 * B * BATCHED_IN * BATCHED_OUT / us / 1e6, 2)}), flush=True)
    return 0


def ctypes_status(lib, device):
    import ctypes

    out = ctypes.c_uint32()
    lib.m3g_device_status(device, ctypes.byref(out), 0)
    return int(out.value)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=500)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-graph", action="store_true", help="launch each step from the host instead of a CUDA graph")
    ap.add_argument("--decode-mode", choices=("ffn+head", "head-only"), default="ffn+head",
                    help="--workload decode under torchrun: rows split over the ranks (FFN and head, or the head)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the 1B decode tokens/s leg")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched Q4_K 28672x8192 sweep")
    ap.add_argument("--workload", choices=["gemv", "lmhead", "decode", "batched"], default="gemv",
                    help="gemv: Q4_K 14336x4096 GEMV per GPU (the headline, with the decode and batched legs); "
                         "lmhead: Q6_K 128256x4096 rows sharded over the GPUs + all-gather; "
                         "decode: the 1B decode alone (--steps tokens); batched: one Q4_K 28672x8192 GEMM")
    ap.add_argument("--batch", type=int, default=8, help="columns of X for --workload batched")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "lmhead":
        return run_lmhead(args)
    if args.workload == "decode":
        return run_decode(args)
    if args.workload == "batched":
        return run_batched(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
