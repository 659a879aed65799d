"""Shared fixtures for the parity tests: seeded synthetic models, encoder outputs and comparisons."""
from __future__ import annotations

import functools
import json
import os

import numpy as np

from whisper4j_b200 import ggml

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# logits tolerance of the parity contract: max-abs 2e-2 and max-abs relative to the row scale 1e-2
LOGIT_ATOL = 2e-2
LOGIT_RTOL = 1e-2

SMALL = ggml.ModelDimensions(80, 96, 128, 2, 1, 1000, 64, 128, 2, 2)
SMALL_OPTS = dict(bias_std=0.02, ln_std=0.1, std=0.05)


@functools.lru_cache(maxsize=None)
def model_bytes(dims: ggml.ModelDimensions, seed: int, wtype: str = "f16", opts: tuple = ()) -> bytes:
    return ggml.synthetic_model_bytes(dims, seed, wtype, **dict(opts))


@functools.lru_cache(maxsize=None)
def parsed(dims, seed, wtype="f16", opts=()):
    return ggml.parse(model_bytes(dims, seed, wtype, opts))


def encoder_output(seed: int, n_audio_ctx: int, d: int) -> np.ndarray:
    """Seeded stand-in for the encoder output (rows standardised like ln_post with gamma=1, beta=0)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n_audio_ctx, d), dtype=np.float32)
    x = (x - x.mean(axis=1, keepdims=True)) / x.std(axis=1, keepdims=True)
    return x.astype(np.float32)


def load_golden(name):
    with open(os.path.join(GOLDEN, f"decode_steps_{name}.json")) as f:
        return json.load(f)


def assert_logits_close(got, want, atol=LOGIT_ATOL, rtol=LOGIT_RTOL, what="logits"):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    err = np.abs(got - want)
    scale = max(float(np.abs(want).max()), 1e-6)
    assert float(err.max()) <= atol, f"{what}: max |diff| {err.max():.3e} > {atol}"
    assert float(err.max()) / scale <= rtol, f"{what}: max |diff| / max |ref| {err.max() / scale:.3e} > {rtol}"


def first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None if len(a) == len(b) else min(len(a), len(b))


def oracle_prefix_scores(ora, xa, prompt, seq, suppress, eot, ts_begin=-1, logits=None):
    """Beam scores of every prefix of `seq` under the oracle: the running sum of the processed
    log-softmax the reference's decodeBeam ranks candidates by (WhisperDecoder.java:236-330:
    suppressBlank at step 0, the suppress list, the n-gram block and timestamp rules after it)."""
    from oracle import oracle as O
    seq = list(seq)
    if logits is None:  # else: the oracle's logits of prompt + seq[:-1] (teacher forced), one row each
        logits = ora.forward(list(prompt) + seq[:-1], xa, None)
    logits = logits[len(prompt) - 1:]
    out, total = [], 0.0
    for i, tok in enumerate(seq):
        row = np.array(logits[i], np.float32)
        if i == 0:
            row[eot] = -np.inf
            if row.size > 220:
                row[220] = -np.inf
        row[list(suppress)] = -np.inf
        if i > 0:
            row = O.apply_repetition_penalty(row, seq[:i])
            if ts_begin > 0:
                row = O.apply_timestamp_rules(row, seq[:i], ts_begin, eot, False)
        r64 = row.astype(np.float64)
        mx = r64.max()
        lse = mx + np.log(np.exp(r64 - mx).sum())
        total += float(np.float32(r64[tok] - lse))
        out.append(total)
    return out


def check_beam(got, want, ora, xa, prompt, suppress, eot, beam, max_tokens, ts_begin=-1, tol=LOGIT_ATOL):
    """Beam-search ids equal to the oracle's, or a near tie where they part.

    ``want`` is the oracle's decode_beam(..., trace=True).  The GPU's sequence is followed through
    the oracle's kept beams step by step; at the first step where the oracle did not keep its prefix,
    the prefix's oracle score must be within ``tol`` of the step's cut (the lowest kept score), i.e.
    the two searches split at a near tie of ranked candidate scores.  If the oracle kept every prefix,
    the final length-normalised pick must be a near tie instead."""
    g = list(got)
    if g == list(want["tokens"]):
        return "equal"
    tr = want["trace"]
    finished = len(g) < max_tokens  # a sequence shorter than max_tokens ended with an eot candidate
    seq_for_scores = g + ([eot] if finished else [])
    scores = oracle_prefix_scores(ora, xa, prompt, seq_for_scores, suppress, eot, ts_begin)
    beams, cut = {}, {}
    for s in sorted({int(r[0]) for r in tr}):
        rows = tr[tr[:, 0] == s]
        kept = {}
        for _, par, tok, sc, out in rows:
            if out >= 0:
                seq = (int(tok),) if s == 0 else beams[s - 1][int(par)][0] + (int(tok),)
                kept[int(out)] = (seq, float(sc))
        if not kept:
            break
        nb = [kept[i] for i in sorted(kept)]
        cut[s] = min(sc for _, sc in nb)
        while len(nb) < beam:
            nb.append(nb[0])
        beams[s] = nb
    for s in range(len(g)):
        if s not in beams:
            break
        if tuple(g[:s + 1]) in {q for q, _ in beams[s]}:
            continue
        gap = cut[s] - scores[s]
        assert gap < tol, f"beam split at step {s}: the GPU kept a prefix the oracle scores {gap:.3e} below its cut"
        return f"near tie at step {s} ({gap:.2e})"
    g_norm = scores[-1] / max(len(g), 1)
    w_norm = want["sum_logprob"] / max(len(want["tokens"]), 1)
    assert w_norm - g_norm < tol, f"final pick: oracle {w_norm:.5f} vs GPU sequence {g_norm:.5f}"
    return f"near tie in the final pick ({w_norm - g_norm:.2e})"


def needs_fallback_ref(r):
    """WhisperDecoder.needsFallback (WhisperDecoder.java:435-440), on a DecodeResult."""
    if r.compression_ratio > 2.4:
        return not (r.no_speech_prob > 0.6 and r.avg_logprob < -1.0)
    return r.avg_logprob < -1.0 and not (r.no_speech_prob > 0.6)


def fallback_policy_ref(attempt):
    """WhisperDecoder.decodeWithFallback (WhisperDecoder.java:119-149): attempt(temperature) -> DecodeResult.
    Returns (result, temperature, attempts made)."""
    best, best_t, n = None, None, 0
    for temp in (0.0, 0.2, 0.4, 0.6, 0.8, 1.0):
        r = attempt(temp)
        n += 1
        if not needs_fallback_ref(r):
            return r, temp, n
        if best is None or r.avg_logprob > best.avg_logprob:
            best, best_t = r, temp
        if temp == 0.0 and r.compression_ratio <= 2.4:
            break
        if temp > 0.0 and r.avg_logprob < best.avg_logprob - 1.0:
            break
    return best, best_t, n
