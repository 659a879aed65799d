#!/usr/bin/env python3
"""Benchmark of the B200 Whisper decoder token loop (libwhisper4j_cuda.so).

One bench step = one full decode call over this rank's streams (prompt + forced
max_tokens tokens per stream), i.e. the work WhisperDecoder.decode / decodeBeam does
for its 30 s chunks.  The default workload is the largest single-GPU configuration of the
benchmark list: large-v3-turbo, 256 independent streams, greedy, 224 forced tokens, the
streams sharded over the GPUs of the run (strong scaling: 256 / N streams per GPU; streams
are independent, so there is no collective on the data path).  Batch-1 latency of the same
model is reported beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU restatement of the
reference's Java decoder (oracle/, single-threaded per stream like the reference) on the
host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from whisper4j_b200 import ggml  # noqa: E402

# name -> workload (the benchmark configurations).  "streams" is per GPU (weak scaling);
# "streams_total" is the job's total, sharded over the GPUs (strong scaling).
CONFIGS = {
    "turbo-greedy-256": dict(arch="large-v3-turbo", wtype="f16", beam=1, max_tokens=224, streams_total=256,
                             note="configs[3]: large-v3-turbo, 256 streams sharded over the GPUs, greedy, "
                                  "224 forced tokens"),
    "base.en-beam5": dict(arch="base.en", wtype="f16", beam=5, max_tokens=224, streams=1,
                          note="configs[1]: base.en, beam 5, 224 forced tokens, 1 stream per GPU"),
    "tiny.en-greedy": dict(arch="tiny.en", wtype="f16", beam=1, max_tokens=64, streams=1,
                           note="configs[0]: tiny.en, greedy, batch 1, 64 forced tokens"),
    "small-greedy-64": dict(arch="small", wtype="f16", beam=1, max_tokens=128, streams=64,
                            note="configs[2]: small, 64 streams per GPU, greedy, 128 forced tokens"),
    "turbo-greedy-b1": dict(arch="large-v3-turbo", wtype="f16", beam=1, max_tokens=224, streams=1,
                            note="north star: large-v3-turbo batch 1, greedy, 224 forced tokens"),
    "turbo-greedy-32": dict(arch="large-v3-turbo", wtype="f16", beam=1, max_tokens=224, streams=32,
                            note="configs[3] at 8 GPUs: 256 streams = 32 per GPU, greedy, 224 tokens"),
    "turbo-greedy-128": dict(arch="large-v3-turbo", wtype="f16", beam=1, max_tokens=224, streams=128,
                             note="configs[3] at 2 GPUs: 256 streams = 128 per GPU, greedy, 224 tokens"),
    "turbo-greedy-64": dict(arch="large-v3-turbo", wtype="f16", beam=1, max_tokens=224, streams=64,
                            note="configs[3] at 4 GPUs: 256 streams = 64 per GPU, greedy, 224 tokens"),
    "large-v3-q8-beam5": dict(arch="large-v3", wtype="q8_0", beam=5, max_tokens=444, streams=1,
                              note="configs[4] per stream: large-v3 Q8_0, beam 5, 448-position context"),
}
DEFAULT_CONFIG = "turbo-greedy-256"
MODEL_SEED = 1234


def prompt_for(dims):
    # the 4-token SOT prompt: ids of sot, language, task, notimestamps roles for this vocabulary
    if dims.n_vocab >= 51865:
        return [50258, 50259, 50360, 50364] if dims.n_vocab == 51866 else [50258, 50259, 50359, 50363]
    return [50257, 50258, 50259, 50362]


def eot_for(dims):
    return 50257 if dims.n_vocab >= 51865 else 50256


def encoder_output(seed, n_audio_ctx, d):
    """Seeded stand-in for the encoder output: rows standardised like ln_post (gamma 1, beta 0)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n_audio_ctx, d), dtype=np.float32)
    x = (x - x.mean(axis=1, keepdims=True)) / x.std(axis=1, keepdims=True)
    return x.astype(np.float32)


def step_bytes(dims, wtype, streams, beam, max_tokens, n_prompt):
    """Algorithmic HBM bytes of one token step: weights + cross K/V per stream + self K/V per sequence."""
    d, L, V = dims.n_text_state, dims.n_text_layer, dims.n_vocab
    wbytes = 2.0 if wtype == "f16" else 34.0 / 32.0
    W = 14.0 * d * d * L * wbytes + V * d * 2.0
    X = 2.0 * dims.n_audio_ctx * d * L * 2.0
    t_mean = n_prompt + max_tokens / 2.0
    Q = streams * beam
    return W + streams * X + Q * (2.0 * t_mean * d * L * 2.0 + 2.0 * d * L * 2.0), W


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, gpu_index=0):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                if int(p[0]) != gpu_index and len({q.split(",")[0] for q in self.lines}) > 1:
                    continue
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (restatement of the reference's scalar Java decoder)
# ---------------------------------------------------------------------------
def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def shard(cfg, rank, world):
    """Global stream ids of this rank, the job's total and the scaling kind.  A strong-scaling
    workload deals its streams round-robin over the ranks (stream i -> rank i mod world, as
    whisper4j_b200.shard does); a weak-scaling one gives every rank the same count."""
    if "streams_total" in cfg:
        total = cfg["streams_total"]
        return [i for i in range(total) if i % world == rank], total, "strong"
    per = cfg["streams"]
    return [rank * per + i for i in range(per)], per * world, "weak"


def cpu_decode_sample(gm, dims, cfg, stream_ids, sample_steps):
    """Decode `sample_steps` steps of each stream, one oracle thread per stream at a time (the
    reference's decoder is single-threaded per call and thread-safe across calls), with as many
    threads as the host has cores.  Returns tokens, seconds (slowest thread's token-loop time),
    threads, wall seconds."""
    from oracle import oracle as O
    O.set_threads(1)
    model = O.OracleModel(gm)
    prompt, eot = prompt_for(dims), eot_for(dims)
    n = len(stream_ids)
    threads = max(1, min(n, os.cpu_count() or 1))
    results = [0.0] * n

    def work(idx):
        for k in range(idx, n, threads):
            xa = encoder_output(stream_ids[k], dims.n_audio_ctx, dims.n_text_state)
            if cfg["beam"] > 1:
                r = model.decode_beam(xa, prompt, eot, cfg["max_tokens"], suppress=[eot], beam=cfg["beam"],
                                      max_steps=sample_steps)
            else:
                r = model.decode(xa, prompt, eot, cfg["max_tokens"], suppress=[eot], max_steps=sample_steps)
            results[k] = r["loop_seconds"]

    ts = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    wall = time.perf_counter() - t0
    # per-thread loop seconds run concurrently: the slowest thread bounds the sample
    per_thread = [sum(results[k] for k in range(i, n, threads)) for i in range(threads)]
    tokens = n * (sample_steps - 1) * cfg["beam"]
    return tokens, max(per_thread), threads, wall


def run_reference(args, cfg, dims, rank, world):
    """The reference arm: the oracle port of the reference's CPU decoder (the Java reference needs a
    JDK, which this image lacks) on the host cores, one stream per thread, every core busy.  Each
    bench step decodes a bounded sample of the workload's streams (as many as there are cores)
    for a few token steps; tokens/s counts the token loop after the prompt, as the GPU arm does."""
    if rank != 0:
        return 0
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, MODEL_SEED, cfg["wtype"]))
    _, total, scaling = shard(cfg, 0, world)
    n_sample = max(1, min(total, os.cpu_count() or 1))
    sample = int(os.environ.get("W4J_REF_SAMPLE_STEPS", "0")) or max(3, min(12, int(12 / cfg["beam"]) + 2))
    times, toks = [], 0
    threads = 1
    for i in range(args.warmup + args.steps):
        ids = [(i * n_sample + k) % total for k in range(n_sample)]
        t, sec, threads, _ = cpu_decode_sample(gm, dims, cfg, ids, sample)
        if i >= args.warmup:
            times.append(sec)
            toks += t
    value = toks / sum(times)
    out = {"metric": "decoder tokens/s", "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / args.steps,
           "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": args.config, "note": cfg["note"], "model_arch": cfg["arch"],
                      "weights": cfg["wtype"], "streams_total": total, "beam": cfg["beam"],
                      "max_tokens": cfg["max_tokens"]},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                            "cpu_model": cpu_model(),
                            "sample": f"per bench step {n_sample} of the {total} streams, {sample - 1} token steps "
                                      f"each after the prompt (prompt and cross K/V projection excluded), one "
                                      f"stream per thread on {threads} threads; oracle/w4j_oracle.c, the scalar f32 "
                                      f"restatement of WhisperDecoder"},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


# kernel classes of w4j_set_kernel_timing
KCLASSES = {1: "projections", 2: "self-attention", 3: "cross-attention", 4: "vocabulary logits", 5: "token selection"}
KNAMES = {1: "k_gemv / k_gemm_tc", 2: "k_attn / k_attn_pairs (self)", 3: "k_attn_pairs / k_attn_stream / k_attn (cross)",
          4: "k_logits_tc / k_logits", 5: "k_select_*"}


def class_bytes(cls, dims, wtype, S, B, T, n_prompt):
    """Algorithmic HBM bytes per launch of a kernel class at this workload (mean over the
    graph-replayed steps 1 .. T-1, whose self-attention spans n_prompt + 1 .. n_prompt + T - 1 keys)."""
    d, L, V, A = dims.n_text_state, dims.n_text_layer, dims.n_vocab, dims.n_audio_ctx
    M = S * B
    wb = 2.0 if wtype == "f16" else 34.0 / 32.0
    if cls == 1:  # the six projections of a layer: weights + activations in + out (+ residual read)
        proj = [(3 * d, d, 1), (d, d, 2), (d, d, 1), (d, d, 2), (4 * d, d, 1), (d, 4 * d, 2)]
        return sum(N * K * wb + M * K * 4.0 + M * N * 4.0 * f for N, K, f in proj) / 6
    if cls == 2:  # every sequence's self K/V rows + q in + out
        kv = n_prompt + T / 2.0
        return M * 2.0 * kv * d * 2.0 + 2.0 * M * d * 4.0
    if cls == 3:  # every stream's cross K/V of one layer (shared by its beams) + q in + out
        return S * 2.0 * A * d * 2.0 + 2.0 * M * d * 4.0
    if cls == 4:  # the embedding per launch (one launch per chunk of <= 32 rows) + the rows
        chunks = (M + 31) // 32
        return V * d * 2.0 + M * d * 4.0 / chunks
    return M * 148 * 144.0  # selection: the per-block partial records


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, cfg, dims, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from whisper4j_b200.decoder import WhisperDecoder

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ids, total, scaling = shard(cfg, rank, world)
    S, B, T = len(ids), cfg["beam"], cfg["max_tokens"]
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, MODEL_SEED, cfg["wtype"]))
    prompt, eot = prompt_for(dims), eot_for(dims)
    dec = WhisperDecoder(gm, device=local_rank, max_streams=max(S, 1), max_beam=B)
    pinned = [torch.from_numpy(encoder_output(g, dims.n_audio_ctx, dims.n_text_state)).pin_memory() for g in ids]
    for s in range(S):
        dec.set_encoder_output(pinned[s].numpy(), slot=s)
    slots = list(range(S))
    prompts = [prompt] * S
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2

    def one_step(sl=None):
        sl = slots if sl is None else sl
        if B > 1:
            return dec.decode_beam_batch(sl, [prompt] * len(sl), eot, T, suppress_tokens=[eot], beam_size=B)
        return dec.decode_batch(sl, [prompt] * len(sl), eot, T, suppress_tokens=[eot])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_step()
    # ---- device-timed region: inputs resident in HBM ----
    sampler = ClockSampler() if rank == 0 else None
    barrier()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    dev_ms, launches = 0.0, 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        flush.fill_(1.0)  # L2 flush between steps (outside the device-timed decode)
        torch.cuda.synchronize()
        res = one_step()
        ms, _, nl = dec.last_timing()
        dev_ms += ms
        launches += nl
    barrier()
    wall = time.perf_counter() - t0
    clocks = sampler.stop(local_rank) if sampler else None
    tokens = sum(len(r.tokens) for r in res) * B * args.steps
    assert all(len(r.tokens) == T for r in res), "forced-length decode produced a short sequence"
    # ---- end to end through the public API: host encoder outputs in, host results out ----
    e2e_steps = max(1, args.steps // 2)
    e2e_s = 0.0
    for _ in range(e2e_steps):
        flush.fill_(1.0)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        for s in range(S):
            dec.set_encoder_output(pinned[s].numpy(), slot=s)
        one_step()
        e2e_s += time.perf_counter() - t1
    # ---- in-chain time of each kernel class (one profiling decode per class, outside the timed region) ----
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = peaks.get("hbm_gbs")
    src = "measured (MEASURED_PEAKS.json hbm_gbs)" if peak else "fallback"
    peak = peak or 6650.0
    chain = {}
    for cls in KCLASSES:
        dec.kernel_timing(cls)
        flush.fill_(1.0)
        torch.cuda.synchronize()
        one_step()
        cms, cn = dec.kernel_times()
        chain[cls] = (cms, cn)
    dec.kernel_timing(0)
    tot_chain = sum(v[0] for v in chain.values()) or 1.0
    dom = max(chain, key=lambda k: chain[k][0])
    dms, dn = chain[dom]
    alg = class_bytes(dom, dims, cfg["wtype"], S, B, T, len(prompt))
    per_launch_ms = dms / max(dn, 1)
    ach = alg / (per_launch_ms * 1e-3) / 1e9
    roof = {"bound": "hbm", "kernel": f"{KNAMES[dom]} ({KCLASSES[dom]})", "achieved": ach, "peak": peak,
            "peak_source": src, "unit": "GB/s", "frac": ach / peak, "traffic": None,
            "algorithmic_bytes_per_launch": alg, "launch_ms": per_launch_ms, "launches": dn,
            "timing": "in chain: CUDA events recorded inside the step graphs around every launch of the class, "
                      "over one full decode of the workload",
            "class_share_in_chain": {KCLASSES[k]: v[0] / tot_chain for k, v in chain.items()},
            "class_ms_per_decode": {KCLASSES[k]: v[0] for k, v in chain.items()},
            "class_launches_per_decode": {KCLASSES[k]: v[1] for k, v in chain.items()}}
    # ---- batch-1 latency of the same model (one stream of this context) ----
    b1 = None
    if B == 1:
        for _ in range(3):
            one_step([0])
        b1_ms = []
        for _ in range(5):
            flush.fill_(1.0)
            torch.cuda.synchronize()
            one_step([0])
            b1_ms.append(dec.last_timing()[0])
        b1_step = statistics.median(b1_ms) / T
        b1_bytes, b1_w = step_bytes(dims, cfg["wtype"], 1, 1, T, len(prompt))
        b1 = {"us_per_token_step": b1_step * 1e3, "tokens_per_s": 1e3 / b1_step,
              "bytes_per_token_step": b1_bytes,
              "step_frac": b1_bytes / (b1_step * 1e-3) / 1e9 / peak,
              "weight_frac": b1_w / (b1_step * 1e-3) / 1e9 / peak,
              "timing": "median of 5 decodes of one stream (224 forced tokens), device time, L2 flushed"}
    # ---- gather over ranks ----
    vals = torch.tensor([dev_ms, wall, e2e_s, float(tokens)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        dev_ms, wall, e2e_s = mx[0].item(), mx[1].item(), mx[2].item()
        tokens_all = sm[3].item()
    else:
        tokens_all = float(tokens)
    if rank != 0:
        dec.close()
        return 0
    value = tokens_all / (dev_ms * 1e-3)
    per_token_step_ms = dev_ms / args.steps / T
    bstep, wbytes = step_bytes(dims, cfg["wtype"], S, B, T, len(prompt))
    out = {
        "metric": "decoder tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f16" if cfg["wtype"] == "f16" else "q8_0", "data": "synthetic",
        "config": {"workload": args.config, "note": cfg["note"], "model_arch": cfg["arch"], "weights": cfg["wtype"],
                   "streams_total": total, "streams_per_gpu": S, "beam": B, "max_tokens": T,
                   "prompt_tokens": len(prompt), "l2": "flushed between steps (256 MB write)",
                   "parallelism": f"{world} independent shard(s), no collective on the data path",
                   "encoder_output": "seeded standardised rows (the decode metric starts from the encoder output; "
                                     "the front end is timed separately under front_end)"},
        "us_per_token_step": per_token_step_ms * 1e3,
        "step_roofline": {"bytes_per_token_step": bstep, "weight_bytes": wbytes,
                          "achieved_gbs": bstep / (per_token_step_ms * 1e-3) / 1e9,
                          "frac": bstep / (per_token_step_ms * 1e-3) / 1e9 / peak,
                          "weight_frac": wbytes / (per_token_step_ms * 1e-3) / 1e9 / peak},
        "wall_s_timed": wall,
        "e2e": {"value": tokens_all / args.steps * e2e_steps / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": S * dims.n_audio_ctx * dims.n_text_state * 4 + S * len(prompt) * 4,
                "d2h_bytes_per_step": S * (T * 4 + 4 + 8 + 4 + 4 + 4),
                "includes": "w4j_set_encoder_output per stream (pinned host xa -> device, cross K/V projection) "
                            "+ decode + results to host, wall clock"},
        "gpu_launches": launches,
        "clocks": clocks,
        "roofline": roof,
    }
    if b1:
        out["batch1"] = b1
    if world == 1 and not args.no_front_end:
        out["front_end"] = front_end_timing(cfg, local_rank, peaks.get("bf16_tflops"))
    if world == 1 and not args.no_cpu_baseline:
        sample = int(os.environ.get("W4J_CPU_SAMPLE_STEPS", "0")) or max(4, min(24, int(24 / B) + 2))
        ctoks, csec, cthreads, _ = cpu_decode_sample(gm, dims, cfg, [0], sample)
        out["cpu_baseline"] = {"value": ctoks / csec, "unit": "tokens/s", "cores": cthreads, "kind": "port",
                               "cpu_model": cpu_model(),
                               "sample": f"{sample - 1} token steps of one stream after the prompt (prompt and "
                                         f"cross K/V projection excluded), oracle/w4j_oracle.c scalar f32 "
                                         f"restatement of WhisperDecoder, 1 thread"}
    print(json.dumps(out), flush=True)
    dec.close()
    return 0


def seeded_audio(seed: int, seconds: float = 30.0, sr: int = 16000) -> np.ndarray:
    """Three sinusoids with seeded frequencies in [100, 4000] Hz at amplitude 0.1 plus N(0, 0.01) noise."""
    rng = np.random.Generator(np.random.PCG64(seed))
    t = np.arange(int(seconds * sr), dtype=np.float64) / sr
    freqs = rng.uniform(100.0, 4000.0, 3)
    x = sum(0.1 * np.sin(2 * np.pi * f * t) for f in freqs) + rng.normal(0.0, 0.01, t.shape)
    return x.astype(np.float32)


def encoder_flops(dims) -> float:
    """Algorithmic flops of one encoder window: the two convolutions, per block the four projections
    (q / k / v, out, mlp.0, mlp.2) and the attention products (q k^T and p v over all frames)."""
    d, T, L, nm = dims.n_audio_state, dims.n_audio_ctx, dims.n_audio_layer, dims.n_mels
    conv = 2.0 * (2 * T) * d * (3 * nm) + 2.0 * T * d * (3 * d)
    block = 2.0 * T * (3 * d * d + d * d + 8 * d * d) + 4.0 * T * T * d
    return conv + L * block


def front_end_timing(cfg, local_rank, tc_peak):
    """One 30 s window through the device front end (w4j_encode_audio: audio upload, log-mel, encoder,
    cross K/V of a stream) on the workload's architecture with encoder weights; wall clock per window
    after warm-up, the log-mel alone, and the encoder's algorithmic throughput."""
    import torch

    from whisper4j_b200.decoder import WhisperDecoder

    dims = ggml.ARCHS[cfg["arch"]]
    if cfg["wtype"] != "f16":
        return None
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, MODEL_SEED + 1, include_encoder=True))
    audio = seeded_audio(7)
    with WhisperDecoder(gm, device=local_rank, max_streams=1, max_beam=1) as dec:
        for _ in range(3):
            dec.encode_audio(audio, slot=0, return_output=False)
        ms, mel_ms = [], []
        for _ in range(10):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            dec.encode_audio(audio, slot=0, return_output=False)
            ms.append(1e3 * (time.perf_counter() - t0))
            t0 = time.perf_counter()
            dec.log_mel(audio)
            mel_ms.append(1e3 * (time.perf_counter() - t0))
        # the whole chunked loop (w4j_transcribe) on 120 s of audio, greedy, timestamps on
        long_audio = seeded_audio(8, seconds=120.0)
        sot = prompt_for(dims)[:3]
        eot = eot_for(dims)
        # previous-text marker, no-speech, no-timestamps and the first timestamp of this vocabulary
        sot_prev, no_speech, no_ts, ts_begin = {51866: (50362, 50363, 50364, 50365),
                                                 51865: (50361, 50362, 50363, 50364)}.get(
            dims.n_vocab, (50360, 50361, 50362, 50363))
        dec.transcribe(long_audio[:480000], sot, eot, no_speech, no_ts, sot_prev, ts_begin=ts_begin,
                       suppress_tokens=[eot])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        segs, windows = dec.transcribe(long_audio, sot, eot, no_speech, no_ts, sot_prev, ts_begin=ts_begin,
                                       suppress_tokens=[eot])
        tr_s = time.perf_counter() - t0
    w = statistics.median(ms)
    fl = encoder_flops(dims)
    return {"model": cfg["arch"], "window_s": 30, "ms_per_window": w, "log_mel_ms": statistics.median(mel_ms),
            "encoder_flops": fl, "achieved_tflops": fl / (w * 1e-3) / 1e12,
            "frac_of_bf16_peak": fl / (w * 1e-3) / 1e12 / tc_peak if tc_peak else None,
            "includes": "w4j_encode_audio wall clock: 30 s of host audio to the device, log-mel, encoder, the "
                        "stream's cross K/V projection; log_mel_ms: w4j_log_mel with the spectrogram back to the host",
            "data": "seeded sinusoid audio, seeded synthetic weights",
            "transcribe": {"audio_s": 120.0, "wall_s": tr_s, "realtime_factor": 120.0 / tr_s, "windows": windows,
                           "segments": len(segs),
                           "includes": "w4j_transcribe: audio upload, per 30 s window log-mel, encoder, cross K/V, "
                                       "decode with temperature fallback, segments and seek, token ids to the host"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-front-end", action="store_true", help="skip the log-mel + encoder window timing")
    ap.add_argument("--max-tokens", type=int, default=0,
                    help="override the config's forced length (short profiling cases; reported in config)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.max_tokens > 0:
        cfg["max_tokens"] = args.max_tokens
    dims = ggml.ARCHS[cfg["arch"]]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        print(json.dumps({"error": f"--gpus {args.gpus} but WORLD_SIZE is {world}: launch N ranks with torchrun "
                                   f"for --gpus N"}), flush=True)
        return 2
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, cfg, dims, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, cfg, dims, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
