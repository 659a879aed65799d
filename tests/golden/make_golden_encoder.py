#!/usr/bin/env python3
"""Generate golden audio-encoder vectors from the reference's own Python restatement.

Run where a checkout of the reference is available; its path is given with --reference.  It
imports the reference's ``tools/generate_reference_values.py`` (``load_ggml``, ``conv1d``,
``gelu``, ``layer_norm``, ``linear`` and ``mha``: the numpy restatement of WhisperEncoder.forward
that the reference uses to produce stage-by-stage values for cross-validation with Java), feeds it
a seeded synthetic GGML model with encoder tensors (``whisper4j_b200.ggml``) and a seeded log-mel
input, and records per stage the first 8 values and sums, plus every n-th row of the encoder
output (n per case).

The numpy restatement uses the exact tanh GELU where the Java encoder uses its f16-indexed GELU
table (Tensor.gelu, Tensor.java:504-520); that is the one expected difference, and the tests allow
for it.  Fixtures are small JSON files; model and input are regenerated from their seeds.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from whisper4j_b200 import ggml  # noqa: E402

# name -> (dims, model seed, mel seed, extra synthetic options, every how many output rows are kept)
CASES = {
    "enc_small": (ggml.ModelDimensions(80, 96, 128, 2, 2, 1000, 64, 128, 2, 1), 31, 32,
                  dict(bias_std=0.02, ln_std=0.1, std=0.05), 8),
    "enc_tiny": (ggml.ARCHS["tiny.en"], 41, 42, dict(), 100),
}


def mel_input(seed: int, n_mels: int, frames: int) -> np.ndarray:
    """Seeded stand-in for a normalised log-mel spectrogram ((log10 + 4) / 4 lies in about [-1, 1.5])."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.uniform(-1.0, 1.5, (n_mels, frames)).astype(np.float32)


def stage(a: np.ndarray) -> dict:
    a = np.asarray(a, dtype=np.float64)
    return {"shape": list(a.shape), "first8": [float(v) for v in a.ravel()[:8]], "sum": float(a.sum()),
            "abs_sum": float(np.abs(a).sum())}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of sparrowlogic/whisper4j (its tools/ directory)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "tools"))
    import generate_reference_values as ref  # the reference's numpy restatement

    for name, (dims, mseed, xseed, opts, row_step) in CASES.items():
        buf = ggml.synthetic_model_bytes(dims, mseed, include_encoder=True, **opts)
        with tempfile.NamedTemporaryFile(suffix=".bin", delete=False) as f:
            f.write(buf)
            path = f.name
        try:
            W, hp, _ = ref.load_ggml(path)
        finally:
            os.unlink(path)
        mel = mel_input(xseed, dims.n_mels, 2 * dims.n_audio_ctx)
        out = {"dims": list(dataclasses.astuple(dims)), "model_seed": mseed, "mel_seed": xseed, "synthetic": opts,
               "row_step": row_step, "stages": {}}
        # the reference script's stages 2-6 (generate_reference_values.py main), on this model and input
        c1 = ref.gelu(ref.conv1d(mel.reshape(1, dims.n_mels, -1), W["encoder.conv1.weight"],
                                 W["encoder.conv1.bias"].flatten(), stride=1, padding=1))
        out["stages"]["conv1_gelu"] = stage(c1)
        c2 = ref.gelu(ref.conv1d(c1, W["encoder.conv2.weight"], W["encoder.conv2.bias"].flatten(), stride=2,
                                 padding=1))
        out["stages"]["conv2_gelu"] = stage(c2)
        x = c2.transpose(0, 2, 1) + W["encoder.positional_embedding"]
        out["stages"]["pos_embed"] = stage(x)
        for i in range(dims.n_audio_layer):
            bp = f"encoder.blocks.{i}."
            ln = ref.layer_norm(x, W[bp + "attn_ln.weight"], W[bp + "attn_ln.bias"])
            x = x + ref.mha(ln, None, W, bp + "attn.", dims.n_audio_head)
            ml = ref.layer_norm(x, W[bp + "mlp_ln.weight"], W[bp + "mlp_ln.bias"])
            x = x + ref.linear(ref.gelu(ref.linear(ml, W[bp + "mlp.0.weight"], W[bp + "mlp.0.bias"])),
                               W[bp + "mlp.2.weight"], W[bp + "mlp.2.bias"])
            if i == 0:
                out["stages"]["encoder_block0"] = stage(x)
        enc = ref.layer_norm(x, W["encoder.ln_post.weight"], W["encoder.ln_post.bias"])[0]
        out["stages"]["encoder_output"] = stage(enc)
        out["rows"] = {str(r): [float("%.7g" % v) for v in enc[r]] for r in range(0, enc.shape[0], row_step)}
        with open(os.path.join(args.out, f"encoder_{name}.json"), "w") as f:
            json.dump(out, f)
        print(name, "written", enc.shape)


if __name__ == "__main__":
    main()
