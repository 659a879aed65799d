#!/usr/bin/env python3
"""Benchmark of the B200 Whisper decoder token loop (libwhisper4j_cuda.so).

One bench step = one full decode call over this rank's streams (prompt + forced
max_tokens tokens per stream), i.e. the work WhisperDecoder.decode / decodeBeam does
for one 30 s chunk.  The default workload is the configuration the headline metric is
quoted on (base.en, beam 5, 224 forced tokens, one stream per GPU); more streams or
GPUs are weak scaling (streams are independent: no collective on the data path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU restatement of the
reference's Java decoder (oracle/, single-threaded per stream like the reference) on the
host cores instead.
"""
from __future__ import annotations

import argparse
import ctypes
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

# name -> workload (the BASELINE configurations; streams are per GPU, weak scaling)
CONFIGS = {
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
    "large-v3-q8-beam5": dict(arch="large-v3", wtype="q8_0", beam=5, max_tokens=444, streams=1,
                              note="configs[4] per stream: large-v3 Q8_0, beam 5, 448-position context"),
}
DEFAULT_CONFIG = "base.en-beam5"
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


# DRAM bytes per k_gemv launch (read + write, mean over the six projections of a layer) from the
# ncu capture summarised in profiles/k_gemv_base.en-beam5.md; other workloads were not captured.
GEMV_TRAFFIC = {"base.en-beam5": (2.265 + 2.218 + 1.666 + 0.614 + 0.609 + 0.615) / 6 * 1e6}


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
def cpu_decode_sample(gm, dims, cfg, n_streams, sample_steps, seed0=0):
    """Decode `sample_steps` steps of `n_streams` streams, one oracle thread per stream (the reference's
    decoder is single-threaded per call and thread-safe across calls).  Returns tokens, seconds, threads."""
    from oracle import oracle as O
    model = O.OracleModel(gm)
    prompt, eot = prompt_for(dims), eot_for(dims)
    threads = max(1, min(n_streams, os.cpu_count() or 1))
    results = [None] * n_streams
    xas = [encoder_output(seed0 + s, dims.n_audio_ctx, dims.n_text_state) for s in range(n_streams)]

    def work(idx):
        for s in range(idx, n_streams, threads):
            if cfg["beam"] > 1:
                r = model.decode_beam(xas[s], prompt, eot, cfg["max_tokens"], suppress=[eot], beam=cfg["beam"],
                                      max_steps=sample_steps)
            else:
                r = model.decode(xas[s], prompt, eot, cfg["max_tokens"], suppress=[eot], max_steps=sample_steps)
            results[s] = r["loop_seconds"]

    ts = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    wall = time.perf_counter() - t0
    # per-thread loop seconds run concurrently: the slowest thread bounds the sample
    per_thread = [sum(results[s] for s in range(i, n_streams, threads)) for i in range(threads)]
    tokens = n_streams * (sample_steps - 1)
    return tokens, max(per_thread), threads, wall


def run_reference(args, cfg, dims, rank, world):
    if rank != 0:
        return 0
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, MODEL_SEED, cfg["wtype"]))
    n_streams = cfg["streams"] * world
    sample = int(os.environ.get("W4J_REF_SAMPLE_STEPS", "0")) or max(3, min(24, int(24 / cfg["beam"]) + 2))
    times, toks = [], 0
    threads = 1
    for i in range(args.warmup + args.steps):
        t, sec, threads, _ = cpu_decode_sample(gm, dims, cfg, n_streams, sample, seed0=100 * i)
        if i >= args.warmup:
            times.append(sec)
            toks += t
    value = toks / sum(times)
    out = {"metric": "decoder tokens/s", "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": args.config, "note": cfg["note"], "model_arch": cfg["arch"],
                      "weights": cfg["wtype"], "streams": n_streams, "beam": cfg["beam"],
                      "max_tokens": cfg["max_tokens"]},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                            "sample": f"{sample - 1} token steps after the prompt of each of {n_streams} stream(s) "
                                      f"per bench step (prompt and cross K/V projection excluded); oracle/w4j_oracle.c, "
                                      f"the scalar f32 restatement of WhisperDecoder, one thread per stream"},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, cfg, dims, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from whisper4j_b200._lib import check, lib
    from whisper4j_b200.decoder import WhisperDecoder

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    S, B, T = cfg["streams"], cfg["beam"], cfg["max_tokens"]
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, MODEL_SEED, cfg["wtype"]))
    prompt, eot = prompt_for(dims), eot_for(dims)
    dec = WhisperDecoder(gm, device=local_rank, max_streams=S, max_beam=B)
    xas = [encoder_output(1000 * rank + s, dims.n_audio_ctx, dims.n_text_state) for s in range(S)]
    pinned = [torch.from_numpy(x).pin_memory() for x in xas]
    for s in range(S):
        dec.set_encoder_output(pinned[s].numpy(), slot=s)
    slots = list(range(S))
    prompts = [prompt] * S
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2

    def one_step():
        if B > 1:
            return dec.decode_beam_batch(slots, prompts, eot, T, suppress_tokens=[eot], beam_size=B)
        return dec.decode_batch(slots, prompts, eot, T, suppress_tokens=[eot])

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
    tokens = sum(len(r.tokens) for r in res) * args.steps
    assert all(len(r.tokens) == T for r in res), "forced-length decode produced a short sequence"
    # ---- end to end through the C ABI with host buffers ----
    e2e_s = 0.0
    for _ in range(max(1, args.steps // 2)):
        flush.fill_(1.0)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        for s in range(S):
            dec.set_encoder_output(pinned[s].numpy(), slot=s)
        one_step()
        e2e_s += time.perf_counter() - t1
    e2e_steps = max(1, args.steps // 2)
    # ---- kernels replayed alone with CUDA events (cold L2), on the stream they are launched on ----
    M = S * B
    d, V = dims.n_text_state, dims.n_vocab
    st = torch.cuda.current_stream()
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = peaks.get("hbm_gbs")
    src = "measured" if peak else "fallback"
    peak = peak or 6650.0

    def time_alone(launch, reps=20):
        # a device-side sleep ahead of the first event keeps the stream busy while the host
        # submits the event pair and the launch, so the events bracket device time only
        durs = []
        for i in range(args.warmup + reps):
            flush.fill_(1.0)
            torch.cuda._sleep(200000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            launch()
            e1.record(st)
            e1.synchronize()
            if i >= args.warmup:
                durs.append(e0.elapsed_time(e1))
        return statistics.median(durs)

    # dominant kernel by time share (profiles/launches_*.md): the projections (k_gemv, or k_gemm_tc
    # from 16 rows on), the six of a decoder layer at this workload's M, K and N (LayerNorm
    # prologue / GELU / residual epilogues)
    from whisper4j_b200._lib import GGML_F16, GGML_Q8_0
    proj = [(3 * d, d, 1, 0), (d, d, 0, 2), (d, d, 1, 0), (d, d, 0, 2), (4 * d, d, 1, 1), (d, 4 * d, 0, 2)]
    gdur, galg = [], []
    for N, K, ln, epi in proj:
        W = (torch.randn(N, K, device=dev) * 0.02).half()
        wt = GGML_F16
        if cfg["wtype"] == "q8_0":
            raw = torch.empty(N * K // 32 * 34, dtype=torch.uint8, device=dev)
            raw.view(-1, 34)[:, 2:] = torch.randint(-127, 128, (N * K // 32, 32), device=dev).to(torch.int8).view(torch.uint8)
            raw.view(-1, 34)[:, :2] = torch.full((N * K // 32, 1), 0.01, device=dev).half().view(torch.uint8)
            W = torch.empty(N * K + N * K // 16, dtype=torch.uint8, device=dev)
            check(lib().w4j_q8_0_repack(vp(raw), N, K, vp(W), ctypes.c_void_p(st.cuda_stream)))
            wt = GGML_Q8_0
        x = torch.randn(M, K, device=dev)
        y = torch.zeros(M, N, device=dev)
        bias = torch.zeros(N, device=dev)
        g, bt = torch.ones(K, device=dev), torch.zeros(K, device=dev)
        gdur.append(time_alone(lambda: check(lib().w4j_op_linear(
            dec._ctx, vp(x), M, K, vp(W), wt, N, vp(bias), vp(g) if ln else None, vp(bt) if ln else None, epi, vp(y),
            ctypes.c_void_p(st.cuda_stream)))))
        wbytes_ = N * K * 2 if cfg["wtype"] == "f16" else N * K * 34 // 32
        galg.append(wbytes_ + M * K * 4 + M * N * 4 * (2 if epi == 2 else 1))
    g_ms, g_alg = sum(gdur) / len(gdur), sum(galg) / len(galg)
    g_ach = g_alg / (g_ms * 1e-3) / 1e9
    # from 16 rows on, f16 projections run on the tcgen05 kernel (w4j_op_linear dispatches as the decoder does)
    kname = "k_gemm_tc (tcgen05, split K over a cluster)" if M >= 16 and cfg["wtype"] == "f16" else "k_gemv"
    roof = {"bound": "hbm", "kernel": kname + ": the six projections of one decoder layer (QKV with LN, attn.out + "
                                      "residual, cross q with LN, cross out + residual, mlp.0 with LN + GELU, "
                                      "mlp.2 + residual), each replayed alone",
            "achieved": g_ach, "peak": peak, "peak_source": src, "unit": "GB/s", "frac": g_ach / peak,
            "traffic": GEMV_TRAFFIC.get(args.config) if not args.max_tokens else None,
            "algorithmic_bytes_per_launch": g_alg, "launch_ms": g_ms,
            "launch_ms_each": gdur, "timing": "cold L2, alone, CUDA events around one launch queued behind a device sleep"}
    roof_logits = None
    if cfg["wtype"] == "f16":
        E = torch.from_numpy(np.frombuffer(gm.tensors["decoder.token_embedding.weight"].data, np.float16).copy()
                             ).to(dev).view(V, d)
        x = torch.randn(M, d, device=dev)
        g = torch.ones(d, device=dev)
        bta = torch.zeros(d, device=dev)
        tok = torch.zeros(M, dtype=torch.int32, device=dev)
        lp = torch.zeros(M, dtype=torch.float64, device=dev)
        kern_ms = time_alone(lambda: check(lib().w4j_op_logits_argmax(
            dec._ctx, vp(x), M, vp(E), V, vp(g), vp(bta), vp(tok), vp(lp), ctypes.c_void_p(st.cuda_stream))))
        alg = V * d * 2.0 + M * d * 4.0
        achieved = alg / (kern_ms * 1e-3) / 1e9
        roof_logits = {"bound": "hbm", "kernel": "k_logits_tc (vocabulary logits + processors + partial reductions) "
                                                 "followed by the argmax merge", "achieved": achieved, "peak": peak,
                       "peak_source": src, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                       "algorithmic_bytes_per_launch": alg, "launch_ms": kern_ms,
                       "timing": "cold L2, alone, CUDA events around one launch queued behind a device sleep"}
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
        return 0
    value = tokens_all / (dev_ms * 1e-3)
    per_token_step_ms = dev_ms / args.steps / T
    bstep, wbytes = step_bytes(dims, cfg["wtype"], S, B, T, len(prompt))
    out = {
        "metric": "decoder tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16" if cfg["wtype"] == "f16" else "q8_0", "data": "synthetic",
        "config": {"workload": args.config, "note": cfg["note"], "model_arch": cfg["arch"], "weights": cfg["wtype"],
                   "streams_per_gpu": S, "beam": B, "max_tokens": T, "prompt_tokens": len(prompt),
                   "l2": "flushed between steps (256 MB write)", "parallelism": f"{world} independent shard(s)",
                   "encoder_output": "seeded standardised rows (encoder out of scope)"},
        "us_per_token_step": per_token_step_ms * 1e3,
        "step_roofline": {"bytes_per_token_step": bstep, "weight_bytes": wbytes,
                          "achieved_gbs": bstep / (per_token_step_ms * 1e-3) / 1e9,
                          "frac": bstep / (per_token_step_ms * 1e-3) / 1e9 / peak,
                          "weight_frac": wbytes / (per_token_step_ms * 1e-3) / 1e9 / peak},
        "wall_s_timed": wall,
        "e2e": {"value": tokens_all / args.steps * e2e_steps / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": S * dims.n_audio_ctx * d * 4 + S * len(prompt) * 4,
                "d2h_bytes_per_step": S * (T * 4 + 4 + 8 + 4 + 4 + 4),
                "includes": "w4j_set_encoder_output (host xa -> device, cross K/V projection) + decode + results"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    out["roofline"] = roof
    if roof_logits:
        out["roofline_logits"] = roof_logits
    if world == 1 and not args.no_cpu_baseline:
        sample = int(os.environ.get("W4J_CPU_SAMPLE_STEPS", "0")) or max(4, min(64, int(40 / B) + 2))
        ctoks, csec, cthreads, _ = cpu_decode_sample(gm, dims, cfg, 1, sample)
        out["cpu_baseline"] = {"value": ctoks / csec, "unit": "tokens/s", "cores": cthreads, "kind": "port",
                               "sample": f"{sample - 1} token steps of one stream after the prompt (prompt and "
                                         f"cross K/V projection excluded), oracle/w4j_oracle.c scalar f32 "
                                         f"restatement of WhisperDecoder, 1 thread"}
    print(json.dumps(out), flush=True)
    dec.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
