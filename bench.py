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
region).  Under torchrun the same GEMV is row-sharded over the ranks and each
step ends with one in-place NCCL all-gather of the fp32 slices (strong
scaling: the total work per step is one whole GEMV); the time is the max over
ranks, and every rank checks the gathered y against the oracle.

The line also carries the vocab-head GEMV (Q6_K 128256 x 4096, sharded the
same way), the batched tcgen05 sweep, and the second half of the metric,
decode tokens/s: greedy decode of a Llama-3.2-1B-shaped model (Q4_K_M mix)
through the device-resident engine, 128 prompt tokens then 256 generated, with
the C restatement of the reference's CPU forward pass timed beside it.
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
HEAD_IN, HEAD_OUT, HEAD_DTYPE = 4096, 128256, 14
L2_NOTE = "inputs larger than L2 (rotating weight copies, > 3x the cache)"


def algorithmic_bytes(in_dim: int, out_dim: int, dtype: int, batch: int = 1) -> int:
    """Weight bytes + 4*B*in + 4*B*out (each weight byte, x and y touched once)."""
    be, bb = {12: (256, 144), 14: (256, 210), 8: (32, 34), 2: (32, 18)}[dtype]
    return in_dim * out_dim // be * bb + 4 * batch * in_dim + 4 * batch * out_dim


def headline_config() -> dict:
    """The workload description both arms print (the same keys and values)."""
    return {"workload": WORKLOAD, "dtype": "Q4_K", "in_dim": IN_DIM, "out_dim": OUT_DIM, "l2": L2_NOTE}


def measured_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def committed_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu capture of this kernel
    (profiles/traffic.json), with where it came from; None if not captured."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
    except (OSError, ValueError):
        return None, None
    v = d.get(f"{kernel}@{workload}")
    if isinstance(v, dict):
        return v.get("bytes"), v.get("source")
    return v, d.get("_source")


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def host_llc_bytes() -> int:
    """Total last-level cache of the host (sum over distinct L3 instances)."""
    seen, total = set(), 0
    base = "/sys/devices/system/cpu"
    try:
        for cpu in os.listdir(base):
            p = os.path.join(base, cpu, "cache", "index3")
            if not cpu.startswith("cpu") or not os.path.isdir(p):
                continue
            try:
                with open(os.path.join(p, "shared_cpu_list")) as f:
                    key = f.read().strip()
                with open(os.path.join(p, "size")) as f:
                    s = f.read().strip()
            except OSError:
                continue
            if key in seen:
                continue
            seen.add(key)
            mult = {"K": 1024, "M": 1024 ** 2, "G": 1024 ** 3}.get(s[-1:], 1)
            total += int(s.rstrip("KMG")) * mult
    except OSError:
        pass
    return total or 64 * 1024 * 1024


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
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "sampled from the warm-up through the timed region"}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---------------------------------------------------------------- CPU reference timing
def cpu_gemv_timing(threads: int, steps: int, step_s: float, warm_s: float = 2.0, dtype: int = DTYPE,
                    in_dim: int = IN_DIM, out_dim: int = OUT_DIM) -> dict:
    """The oracle's port of the reference AVX2 matvec_q4k on this host's cores.

    Used by both the reference arm and the CPU-baseline leg, so the two time
    the same thing the same way: the weights rotate over enough copies that
    the set is larger than three times the host's last-level cache (as the GPU
    arm rotates past the L2), `warm_s` seconds of untimed GEMVs bring the
    thread pool and clocks up, then `steps` steps of R full GEMVs each (R
    sized so a step takes about `step_s`).  Rate = bytes of all timed GEMVs /
    time of all timed steps."""
    from oracle import oracle as O
    from m3_avm_b200 import synth

    raw = synth.weights(dtype, in_dim, out_dim, seed=1)
    x = synth.activations(in_dim, seed=2)
    n_copies = int(min(16, max(2, math.ceil(3 * host_llc_bytes() / raw.size))))
    copies = [raw] + [raw.copy() for _ in range(n_copies - 1)]
    calls = 0
    t_end = time.perf_counter() + warm_s
    t0 = time.perf_counter()
    while True:
        O.matvec_quant(x, copies[calls % n_copies], dtype, in_dim, out_dim, threads=threads)
        calls += 1
        if time.perf_counter() >= t_end and calls >= 3:
            break
    one = (time.perf_counter() - t0) / calls
    reps = max(1, int(round(step_s / one)))
    per_step = []
    i = 0
    for _ in range(steps):
        t0 = time.perf_counter()
        for _ in range(reps):
            O.matvec_quant(x, copies[i % n_copies], dtype, in_dim, out_dim, threads=threads)
            i += 1
        per_step.append(time.perf_counter() - t0)
    total = sum(per_step)
    per_gemv = total / (steps * reps)
    gbs = algorithmic_bytes(in_dim, out_dim, dtype) / per_gemv / 1e9
    name = {12: "Q4_K", 14: "Q6_K", 8: "Q8_0", 2: "Q4_0"}[dtype]
    kernel = "AVX2 matvec_q4k" if dtype == 12 else "matvec_blocked"
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{steps} steps x {reps} full {out_dim}x{in_dim} {name} GEMVs over {n_copies} rotating weight "
                      f"copies (C restatement of the reference {kernel}, {threads} OpenMP threads) after "
                      f"{warm_s:.0f} s of warm-up; {per_gemv * 1e3:.3f} ms per GEMV over {total:.1f} s",
            "ms_per_gemv": round(per_gemv * 1e3, 4), "gemvs_per_step": reps, "seconds": round(total, 2),
            "per_step_s": per_step}


DECODE_PROMPT, DECODE_GEN = 128, 256


def _decode_run(args, dev, world, shape, tensors, prompt, resume_at: int | None = None) -> dict:
    """One decoder: warm-up, then device-timed generation and the e2e call;
    optionally a cache truncation to `resume_at` positions and a resumed
    generation checked against the first."""
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
    resumed = None
    if resume_at is not None:
        # truncate_kv_cache, then resume from the token at position resume_at:
        # the stream after it must repeat the uninterrupted one
        full = dec.tokens(0, DECODE_PROMPT + DECODE_GEN)
        dec.truncate_kv_cache(resume_at)
        n_more = DECODE_PROMPT + DECODE_GEN - resume_at - 1
        again = dec.generate(full[resume_at:resume_at + 1], n_more)
        resumed = bool(np.array_equal(again, full[resume_at + 1:resume_at + 1 + n_more]))
    dec.close()
    return {"gen_ms": gen_ms, "tok_s": (DECODE_GEN - 1) / (gen_ms / 1e3), "e2e_s": e2e_s, "exchange": exchange,
            "toks": toks, "match": bool((toks == toks2).all()), "resumed_match": resumed}


def decode_leg(args, dev, world: int = 1) -> dict:
    """Greedy decode of the Llama-3.2-1B-shaped model (16 layers, hidden 2048,
    FFN 8192, 32/8 heads x 64, vocab 128256, Q4_K attention/gate/up/embedding,
    Q6_K down and head), seeded synthetic weights: a 128-token prompt, then
    256 generated tokens, all steps device-resident.  Under torchrun the engine
    is row-sharded over the ranks in two ways, both measured: the vocab head
    alone (every rank keeps the layers; the greedy keys merge by peer atomics
    over NVLink, or by one NCCL all-reduce per token where peers cannot be
    mapped) and the FFN plus the head (rows exchanged every layer); the time is
    the max over ranks (strong scaling: one model, one sequence).  Each
    sharded layout's token stream is compared with the single-GPU engine's on
    the same weights (run on rank 0), and again after a cache truncation and
    resume."""
    import torch.distributed as dist

    from m3_avm_b200 import matvec_quant as MQ
    from m3_avm_b200 import model

    shape = model.LLAMA_1B
    tensors = model.synthetic_tensors(shape, seed=1)
    prompt = model.prompt_tokens(shape, DECODE_PROMPT, seed=2)
    resume_at = DECODE_PROMPT + 64
    modes = {}
    if world > 1:
        for name, shard_ffn in (("head-only", 0), ("ffn+head", 1)):
            MQ.set_tuning("decode_shard_ffn", shard_ffn)
            modes[name] = _decode_run(args, dev, world, shape, tensors, prompt, resume_at=resume_at)
        MQ.set_tuning("decode_shard_ffn", 1)
        best = max(modes, key=lambda k: modes[k]["tok_s"])
        r = modes[best]
        # the single-GPU engine on the same weights (rank 0's GPU), broadcast
        ref = [None]
        if dist.get_rank() == 0:
            single = _decode_run(args, dev, 1, shape, tensors, prompt)
            ref = [single["toks"]]
        dist.broadcast_object_list(ref, src=0)
        ok = {k: bool(np.array_equal(v["toks"], ref[0])) for k, v in modes.items()}
        ok_t = torch_all_ranks(all(ok.values()) and all(v["resumed_match"] for v in modes.values()), dev)
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
                            "e2e_tokens_per_s": round(DECODE_GEN / v["e2e_s"], 1),
                            "tokens_match_single_gpu": ok[k],
                            "tokens_match_after_truncate_resume": v["resumed_match"]} for k, v in modes.items()}
        out["matches_single_gpu_all_ranks"] = ok_t
        out["check"] = (f"each layout's 256 generated tokens equal the single-GPU engine's on the same weights "
                        f"(rank 0's GPU), and a truncation to {resume_at} positions then resume repeats the stream; "
                        f"AND over ranks")
    if not args.no_cpu and world == 1:
        out["cpu_baseline"] = cpu_decode_rate(shape, tensors, prompt)
    return out


def torch_all_ranks(flag: bool, dev) -> bool:
    """AND of a per-rank flag over the process group."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=dev)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


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

    threads = host_threads()
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


def run_cpu_table(args) -> int:
    """The reference CPU path of every single-GEMV config on this host (one
    line per config, timed as the CPU-baseline leg)."""
    threads = host_threads()
    out = {}
    for name, (dt, i, o) in {"c0 Q4_K 4096x4096": (12, 4096, 4096), "c1 Q4_K 14336x4096": (12, 4096, 14336),
                             "c1 Q6_K 4096x14336": (14, 14336, 4096), "c1 Q8_0 4096x4096": (8, 4096, 4096),
                             "c2 Q6_K 128256x4096": (14, 4096, 128256)}.items():
        r = cpu_gemv_timing(threads, steps=4, step_s=1.0, warm_s=1.0, dtype=dt, in_dim=i, out_dim=o)
        r.pop("per_step_s", None)
        out[name] = {"gbs": r["value"], "ms_per_gemv": r["ms_per_gemv"], "cores": threads}
    cpu = ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next(l.split(":", 1)[1].strip() for l in f if l.startswith("model name"))
    except (OSError, StopIteration):
        pass
    print(json.dumps({"cpu_table": out, "cpu_model": cpu, "threads": threads}), flush=True)
    return 0


def run_reference(args) -> int:
    """The reference's CPU path of the workload (the oracle's port of the AVX2
    matvec_q4k; the Rust crate cannot be built here) on all host threads.  A
    step is a bounded sample: R full GEMVs, R sized so the run stays within a
    few minutes.  Under torchrun rank 0 alone runs; the others exit."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = host_threads()
    step_s = min(0.5, 150.0 / max(1, args.steps + args.warmup))
    cb = cpu_gemv_timing(threads, args.steps, step_s, warm_s=max(2.0, args.warmup * step_s))
    gbs = cb["value"]
    dt = sum(cb["per_step_s"]) / max(1, args.steps)
    cb.pop("per_step_s")
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": headline_config(),
        "parallelism": "host CPU (rank 0 only)",
        "cpu_baseline": cb,
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "step": f"{cb['gemvs_per_step']} full GEMVs per step",
    }
    if not args.no_decode:
        from m3_avm_b200 import model

        shape = model.LLAMA_1B
        line["decode"] = {"cpu_baseline": cpu_decode_rate(shape, model.synthetic_tensors(shape, seed=1),
                                                          model.prompt_tokens(shape, DECODE_PROMPT, seed=2))}
        line["decode"]["tokens_per_s"] = line["decode"]["cpu_baseline"]["value"]
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- timed replays
class Replayer:
    """K steps over n rotating weight copies, launched from CUDA graphs.

    Step i launches copy i % n.  Launches inside one graph chain with
    programmatic dependent launch; a graph boundary does not, so the timed
    steps sit in as few graphs as possible.  Up to ONE_GRAPH steps, the K
    timed steps are one graph replayed once; the same graph is then replayed
    7 more times, each timed, for a median and best window.  Beyond that the
    timed steps are at most 64 windows of whole cycles (each one replay of one
    graph) plus a remainder, with an event after each.  Every graph the timed
    region replays is captured and replayed twice before it, and ~256 more
    steps of it run right before the timed region, whatever the requested
    warm-up."""

    ONE_GRAPH = 2048

    def __init__(self, step, n: int, stream, dev, use_graph: bool = True):
        import torch

        self.torch = torch
        self.step, self.n, self.stream, self.dev, self.use_graph = step, n, stream, dev, use_graph
        self.cap = torch.cuda.Stream(dev)
        self.graphs: dict = {}
        self.warm_steps = 0

    def plan(self, K: int) -> list[tuple[str, int, int]]:
        """(kind, first step, length) per timed window."""
        n = self.n
        if K <= self.ONE_GRAPH:
            return [("seg", 0, K)]
        cycles = K // n
        per = -(-cycles // 64)
        wins = [("cyc", s, per * n) for s in range(0, (cycles // per) * per * n, per * n)]
        s = (cycles // per) * per * n
        if K > s:
            wins.append(("seg", s, K - s))
        return wins

    def _graph(self, start: int, length: int):
        key = (start % self.n, length)
        g = self.graphs.get(key)
        if g is None:
            g = self.torch.cuda.CUDAGraph()
            with self.torch.cuda.graph(g, stream=self.cap, capture_error_mode="thread_local"):
                for i in range(length):
                    self.step((start + i) % self.n, self.cap)
            self.graphs[key] = g
        return g

    def window(self, kind: str, start: int, length: int) -> None:
        if not self.use_graph:
            for i in range(length):
                self.step((start + i) % self.n, self.stream)
        else:
            self._graph(start, length).replay()

    def warm(self, K: int, W: int) -> None:
        done = 0
        seen = set()
        plan = self.plan(K)
        for kind, s, length in plan:
            key = (s % self.n, length)
            if key in seen:
                continue
            seen.add(key)
            for _ in range(2):
                self.window(kind, s, length)
                done += length
        kind, s, length = plan[0]
        while done < W:
            self.window(kind, s, length)
            done += length
        self.warm_steps = done

    def preroll(self, steps: int) -> None:
        """Untimed replays of the first window, queued right before the timed region."""
        kind, s, length = self.plan_first
        reps = max(1, -(-steps // length))
        for _ in range(reps):
            self.window(kind, s, length)
        self.warm_steps += reps * length

    def timed(self, K: int) -> dict:
        torch = self.torch
        plan = self.plan(K)
        marks = []
        ev0 = torch.cuda.Event(enable_timing=True)
        ev0.record(self.stream)
        for kind, s, length in plan:
            self.window(kind, s, length)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(self.stream)
            marks.append((ev, length))
        extra = 7 if len(plan) == 1 else 0  # more replays of the same K-step graph, after the timed region
        for _ in range(extra):
            kind, s, length = plan[0]
            self.window(kind, s, length)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(self.stream)
            marks.append((ev, length))
        torch.cuda.synchronize(self.dev)
        ms = ev0.elapsed_time(marks[len(plan) - 1][0])
        prev, win_us = ev0, []
        for ev, length in marks:
            win_us.append(prev.elapsed_time(ev) * 1e3 / length)
            prev = ev
        w = {"median_us": round(statistics.median(win_us), 3), "best_us": round(min(win_us), 3),
             "worst_us": round(max(win_us), 3), "windows": len(win_us),
             "steps_per_window": [m[1] for m in marks][:4] + ([] if len(marks) <= 4 else ["..."])}
        if extra:
            w["note"] = ("window 1 is the timed region (all K steps in one graph); windows 2-8 replay the same "
                         "graph right after it")
        return {"ms": ms, "windows": w}

    @property
    def plan_first(self):
        return self._first

    def prepare(self, K: int, W: int) -> None:
        self._first = self.plan(K)[0]
        self.warm(K, W)

    def release(self) -> None:
        self.graphs.clear()


def max_over_ranks(v: float, dev, world: int) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def oracle_check(y: np.ndarray, raw: np.ndarray, dtype: int, in_dim: int, out_dim: int, x: np.ndarray, dev,
                 world: int, threads: int) -> dict:
    """Checker (after the timed region): y against the oracle's port of the
    reference matvec_quant on the same weights, every row within
    1e-5 * ||row||_1 * ||x||_inf; max over ranks and the number of ranks whose
    whole y passes."""
    from oracle import oracle as O

    ref = O.matvec_quant(x, raw, dtype, in_dim, out_dim, threads=threads)
    bound = O.gemv_bound(raw, dtype, in_dim, out_dim, x)
    ratio = float(np.max(np.abs(y.astype(np.float64) - ref.astype(np.float64)) / bound))
    ok = bool(np.isfinite(ratio) and ratio <= 1.0)
    worst = max_over_ranks(ratio, dev, world)
    ranks_ok = int(round(sum_over_ranks(1.0 if ok else 0.0, dev, world)))
    return {"max_err_over_bound": round(worst, 6), "ranks_ok": ranks_ok, "ranks": world,
            "rows_checked_per_rank": out_dim,
            "bound": "per row |y - oracle| <= 1e-5 * ||row||_1 * ||x||_inf"}


def sum_over_ranks(v: float, dev, world: int) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def c_abi_e2e(raw: np.ndarray, dtype: int, in_dim: int, out_dim: int, copies: int, calls: int):
    """us per m3g_offload_matvec call timed by the C program beside the
    library (m3g_e2e_timing): host x in, host y out, weights resident."""
    import tempfile

    from m3_avm_b200 import build_lib

    exe = build_lib.E2E_BIN
    if not os.path.exists(exe):
        return None
    with tempfile.NamedTemporaryFile(suffix=".gguf-blocks", delete=False) as f:
        f.write(raw.tobytes())
        path = f.name
    try:
        r = subprocess.run([exe, path, str(dtype), str(in_dim), str(out_dim), str(copies), str(calls), "50"],
                           capture_output=True, text=True, timeout=300)
    finally:
        os.unlink(path)
    if r.returncode != 0:
        raise RuntimeError("m3g_e2e_timing failed: " + r.stderr[-500:])
    return json.loads(r.stdout.strip().splitlines()[-1])


def _copies_for(l2: int, nbytes: int) -> int:
    return max(2, math.ceil(3 * l2 / max(nbytes, 1)))


def gemv_leg(args, dev, rank: int, world: int, in_dim: int, out_dim: int, dtype: int, seed: int, K: int, W: int,
             sharded_always: bool = False, check: bool = True, e2e_steps: int = 0) -> dict:
    """Time K steps of one GEMV shape (resident weights, rotating copies).

    world == 1 (and not sharded_always): the offload GEMV alone.  Otherwise
    the rows are sharded over the ranks and each step is the local GEMV plus
    one in-place NCCL all-gather of the fp32 slices (m3g_shard_matvec_dev)."""
    import torch
    import torch.distributed as dist

    from m3_avm_b200 import _lib, sharded, synth
    from m3_avm_b200.inference_gpu import GpuOffload

    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    raw = synth.weights(dtype, in_dim, out_dim, seed=seed)
    xh = synth.activations(in_dim, seed=seed + 1)
    x = torch.from_numpy(xh).to(dev)
    stream = torch.cuda.current_stream(dev)
    use_shard = world > 1 or sharded_always
    if use_shard:
        if world > 1:
            s = sharded.ShardedOffload.from_torch_dist(dev.index or 0, in_dim, out_dim, timeout_s=120)
        else:
            s = sharded.ShardedOffload(dev.index or 0, 0, 1, sharded.unique_id(), in_dim, out_dim, timeout_s=120)
        _, rows_local, rpr, _, bytes_local = sharded.shard_plan(dtype, in_dim, out_dim, world, rank)
        n = _copies_for(l2, bytes_local)
        for c in range(n):
            if not s.upload(c, dtype, raw, in_dim, out_dim):
                raise RuntimeError("shard upload failed: " + _lib.last_error())
        y = torch.zeros(s.gather_len(0), dtype=torch.float32, device=dev)

        def step(c, st):
            s.matvec_dev(c, x, y, stream=st.cuda_stream)
    else:
        g = GpuOffload.try_new(in_dim, out_dim, device=dev.index or 0)
        if g is None:
            raise RuntimeError("GpuOffload.try_new failed: " + _lib.last_error())
        bytes_local, rows_local = raw.size, out_dim
        n = _copies_for(l2, bytes_local)
        for c in range(n):
            if not g.upload(c, dtype, raw, in_dim, out_dim):
                raise RuntimeError("upload failed: " + _lib.last_error())
        y = torch.empty(out_dim, dtype=torch.float32, device=dev)

        def step(c, st):
            g.matvec_dev(c, x, y, stream=st.cuda_stream)

    lib = _lib.load()
    rep = Replayer(step, n, stream, dev, use_graph=not args.no_graph)
    rep.prepare(K, W)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    launches0 = int(lib.m3g_launch_count())
    rep.preroll(256)
    t = rep.timed(K)
    host_launches = int(lib.m3g_launch_count()) - launches0
    ms = max_over_ranks(t["ms"], dev, world)
    per_step_s = ms / 1e3 / K
    abytes = algorithmic_bytes(in_dim, out_dim, dtype)
    out = {"per_step_s": per_step_s, "ms": ms, "windows": t["windows"], "weight_copies": n,
           "exchange": s.exchange if use_shard else "single",
           "weight_set_mb": round(n * bytes_local / 2**20, 1), "l2_mb": round(l2 / 2**20, 1),
           "bytes_local": bytes_local, "rows_local": rows_local, "abytes": abytes,
           "warmup_steps_run": rep.warm_steps,
           "gbs": abytes / per_step_s / 1e9, "local_gbs": (bytes_local + 4 * in_dim + 4 * rows_local) / per_step_s / 1e9,
           "gpu_launches": K if not args.no_graph else host_launches}
    rep.release()
    if check:
        torch.cuda.synchronize(dev)
        yh = y.cpu().numpy()[:out_dim]
        out["parity"] = oracle_check(yh, raw, dtype, in_dim, out_dim, xh, dev, world,
                                     threads=max(1, host_threads() // world))
    if e2e_steps:
        # host x in, host y out through the public call (copies in the timed region)
        yo = np.empty(out_dim, np.float32)
        for i in range(min(W, 20)):
            if use_shard:
                s.matvec(i % n, xh, in_dim, out_dim)
            else:
                g.matvec(i % n, xh, in_dim, out_dim, out=yo)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            if use_shard:
                r = s.matvec(i % n, xh, in_dim, out_dim)
            else:
                r = g.matvec(i % n, xh, in_dim, out_dim, out=yo)
            if r is None:
                raise RuntimeError("offload matvec failed: " + _lib.last_error())
        e2e_s = max_over_ranks((time.perf_counter() - t0) / e2e_steps, dev, world)
        out["e2e"] = {"value": round(abytes / e2e_s / 1e9, 3), "unit": "GB/s", "h2d_bytes_per_step": 4 * in_dim,
                      "d2h_bytes_per_step": 4 * out_dim, "us_per_call": round(e2e_s * 1e6, 2), "calls": e2e_steps,
                      "api": ("m3g_shard_matvec (host x/y; local GEMV + NCCL all-gather), called from Python "
                              "ctypes" if use_shard else
                              "m3g_offload_matvec (host x/y, resident weights), called from Python ctypes")}
        if not use_shard:
            c = c_abi_e2e(raw, dtype, in_dim, out_dim, n, max(e2e_steps, 800))
            if c is not None:
                # the C caller's figure is the headline e2e: a Rust caller binds the ABI the same way
                py = dict(out["e2e"])
                out["e2e"] = {"value": round(abytes / (c["us_per_call"] * 1e-6) / 1e9, 3), "unit": "GB/s",
                              "h2d_bytes_per_step": 4 * in_dim, "d2h_bytes_per_step": 4 * out_dim,
                              "us_per_call": c["us_per_call"], "best_window_us_per_call": c["best_window_us_per_call"],
                              "calls": c["calls"],
                              "api": "m3g_offload_matvec (host x/y, resident weights), called from C "
                                     "(m3_avm_b200/e2e_timing.c)",
                              "python_ctypes": {"value": py["value"], "us_per_call": py["us_per_call"],
                                                "calls": py["calls"]}}
    torch.cuda.synchronize(dev)
    if use_shard:
        s.close()
    else:
        g.close()
    return out


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from m3_avm_b200 import _lib

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    peaks, kind = measured_peaks()
    peak = float(peaks["hbm_gbs"])
    sampler = ClockSampler(local)
    sampler.start()

    K, W = args.steps, args.warmup
    e2e_steps = 0 if args.no_e2e else min(K * 10, 5000) if K < 500 else min(K, 5000)
    from m3_avm_b200 import matvec_quant as MQ

    if world > 1:
        MQ.set_tuning("shard_p2p", 0)  # NCCL all-gather first, then the peer stores
    head = gemv_leg(args, dev, rank, world, IN_DIM, OUT_DIM, DTYPE, seed=1, K=K, W=W, e2e_steps=e2e_steps)
    head_modes = None
    if world > 1:
        # the other exchange: rows stored into every rank's region by the GEMV epilogue
        MQ.set_tuning("shard_p2p", 1)
        alt = gemv_leg(args, dev, rank, world, IN_DIM, OUT_DIM, DTYPE, seed=1, K=K, W=W)
        MQ.set_tuning("shard_p2p", 0)
        head_modes = {m["exchange"]: {"us_per_step": round(m["per_step_s"] * 1e6, 3), "gbs": round(m["gbs"], 1),
                                      "parity_ranks_ok": m["parity"]["ranks_ok"]} for m in (head, alt)}
        if alt["per_step_s"] < head["per_step_s"]:
            alt["e2e"] = head.get("e2e")
            head = alt
    clocks = sampler.stop()
    value = head["gbs"]
    per_gpu = head["local_gbs"]
    traffic, traffic_src = committed_traffic("k_gemv_mma", WORKLOAD)
    roofline = {"bound": "hbm", "achieved": round(per_gpu, 2), "peak": peak, "unit": "GB/s",
                "frac": round(per_gpu / peak, 4), "peak_kind": kind,
                "traffic": traffic if world == 1 else None,
                "traffic_source": traffic_src if world == 1 else None,
                "kernel": "k_gemv_mma<MmaQ4K>",
                "algorithmic_bytes_per_launch": head["abytes"] if world == 1 else head["bytes_local"] + 4 * (
                    IN_DIM + head["rows_local"]),
                "timing": ("CUDA events on the launching stream around the timed graph replays; per-launch time = "
                           "window time / launches" if world == 1 else
                           "per GPU: this GPU's rows of the GEMV per step, including the all-gather's time")}

    status = ctypes_status(lib, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_gemv_timing(host_threads(), steps=6, step_s=args.cpu_seconds / 6)
        cpu.pop("per_step_s", None)

    extra = {}
    if not args.no_lmhead:
        lm = gemv_leg(args, dev, rank, world, HEAD_IN, HEAD_OUT, HEAD_DTYPE, seed=11, K=max(K, 20), W=W,
                      sharded_always=True)
        lm_modes = None
        if world > 1:
            from m3_avm_b200 import matvec_quant as MQ

            MQ.set_tuning("shard_p2p", 1)
            lm_alt = gemv_leg(args, dev, rank, world, HEAD_IN, HEAD_OUT, HEAD_DTYPE, seed=11, K=max(K, 20), W=W,
                              sharded_always=True)
            MQ.set_tuning("shard_p2p", 0)
            lm_modes = {m["exchange"]: {"us_per_step": round(m["per_step_s"] * 1e6, 3),
                                        "parity_ranks_ok": m["parity"]["ranks_ok"]} for m in (lm, lm_alt)}
            if lm_alt["per_step_s"] < lm["per_step_s"]:
                lm = lm_alt
            MQ.set_tuning("shard_p2p", -1)  # the library's default again
        extra["lmhead"] = {
            "workload": "q6k_lmhead_128256x4096, rows sharded over the GPUs + all-gather of the fp32 logits (NCCL "
                        "or peer stores, whichever exchange_modes shows faster)", "us_per_step": round(lm["per_step_s"] * 1e6, 2),
            "gbs": round(lm["gbs"], 1), "per_gpu_gbs": round(lm["local_gbs"], 1),
            "frac_of_peak_per_gpu": round(lm["local_gbs"] / peak, 4), "rows_per_gpu": lm["rows_local"],
            "weight_copies": lm["weight_copies"], "windows": lm["windows"], "parity": lm["parity"],
            "parallelism": f"rows{world}+allgather ({lm['exchange']})", "scaling": "strong",
            "exchange_modes": lm_modes}
    if world == 1 and not args.no_orient:
        o = gemv_leg(args, dev, rank, world, OUT_DIM, IN_DIM, DTYPE, seed=21, K=max(K, 20), W=W)
        extra["q4k_4096x14336"] = {
            "workload": "the other orientation the metric string admits: 4096 output rows over 14336 inputs",
            "us_per_step": round(o["per_step_s"] * 1e6, 2), "gbs": round(o["gbs"], 1),
            "frac": round(o["gbs"] / peak, 4), "windows": o["windows"], "parity": o["parity"]}

    decode = None
    if not args.no_decode:
        decode = decode_leg(args, dev, world)
    batched = None
    if not args.no_batched:
        batched = batched_leg(args, dev, rank, world)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(head["ms"] / K, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config(),
            "parallelism": "single GPU" if world == 1 else f"rows{world}+allgather ({head['exchange']})",
            "weight_copies": head["weight_copies"], "weight_set_mb": head["weight_set_mb"], "l2_mb": head["l2_mb"],
            "warmup_steps_run": head["warmup_steps_run"],
            "warmup_note": "every graph the timed region replays is replayed twice first, and 256 more steps run "
                           "right before it; W is the minimum",
            "pct_of_measured_hbm_peak": round(100 * per_gpu / peak, 2),
            "pct_of_8tbps_spec": round(100 * per_gpu / 8000.0, 2),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": head.get("e2e"),
            "gpu_launches": head["gpu_launches"],
            "per_step_windows": head["windows"],
            "parity": head["parity"],
            "exchange_modes": head_modes,
            "timing": "CUDA events around CUDA-graph replays of the steps, max over ranks" if not args.no_graph
                      else "CUDA events around host-launched steps, max over ranks",
            "clocks": clocks,
            "device_status": status,
            **extra,
            "decode": decode,
            "batched": batched,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
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
    ap.add_argument("--steps", type=int, default=20000)
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
    ap.add_argument("--no-lmhead", action="store_true", help="skip the sharded Q6_K vocab-head leg")
    ap.add_argument("--no-orient", action="store_true", help="skip the 4096x14336 orientation (1 GPU)")
    ap.add_argument("--workload", choices=["gemv", "decode", "batched", "cpu-table"], default="gemv",
                    help="gemv: the Q4_K 14336x4096 GEMV (row-sharded + all-gather under torchrun) with the "
                         "lm_head, decode and batched legs; decode: the 1B decode alone (--steps tokens); "
                         "batched: one Q4_K 28672x8192 GEMM; cpu-table: the reference CPU path of every "
                         "single-GEMV config on this host")
    ap.add_argument("--batch", type=int, default=8, help="columns of X for --workload batched")
    ap.add_argument("--tune", action="append", default=[], metavar="KEY=VALUE",
                    help="m3g_set_tuning(KEY, VALUE) before the run (repeatable), e.g. --tune tc8=1")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    for kv in args.tune:
        from m3_avm_b200 import matvec_quant as MQ

        key, _, val = kv.partition("=")
        MQ.set_tuning(key, int(val))
    if args.workload == "cpu-table":
        return run_cpu_table(args)
    if args.workload == "decode":
        return run_decode(args)
    if args.workload == "batched":
        return run_batched(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
