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
