#!/usr/bin/env python3
"""Golden log-mel and encoder stage values from the reference's own stage-by-stage script.

Run where a checkout of the reference is available; its path is given with --reference.  For each
case it writes a seeded synthetic GGML model (``whisper4j_b200.ggml``, encoder tensors included) and a
seeded 30 s 16 kHz mono 16-bit WAV (three sinusoids with seeded frequencies in [100, 4000] Hz at
amplitude 0.1 plus N(0, 0.01) noise), runs the reference's ``tools/generate_reference_values.py
<model> <audio>`` unchanged, and keeps the JSON it prints: per stage (mel, conv1_gelu, conv2_gelu,
pos_embed, encoder_block0, encoder_output, ...) the shape and first 8 values.  The tests regenerate
the audio from the seed (``audio_samples``) and compare.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import wave

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from whisper4j_b200 import ggml  # noqa: E402

# name -> (dims, model seed, audio seed)
CASES = {
    "mel80_tiny": (ggml.ARCHS["tiny.en"], 51, 52),
}


def audio_int16(seed: int, seconds: float = 30.0, sr: int = 16000) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    t = np.arange(int(seconds * sr), dtype=np.float64) / sr
    freqs = rng.uniform(100.0, 4000.0, 3)
    x = sum(0.1 * np.sin(2 * np.pi * f * t) for f in freqs) + rng.normal(0.0, 0.01, t.shape)
    return np.clip(np.round(x * 32767.0), -32768, 32767).astype(np.int16)


def audio_samples(seed: int) -> np.ndarray:
    """The float samples the reference script reads from the WAV (int16 / 32768)."""
    return audio_int16(seed).astype(np.float32) / 32768.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of sparrowlogic/whisper4j (its tools/ directory)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    script = os.path.join(args.reference, "tools", "generate_reference_values.py")
    for name, (dims, mseed, aseed) in CASES.items():
        with tempfile.TemporaryDirectory() as tmp:
            model = os.path.join(tmp, "model.bin")
            with open(model, "wb") as f:
                f.write(ggml.synthetic_model_bytes(dims, mseed, include_encoder=True))
            audio = os.path.join(tmp, "audio.wav")
            with wave.open(audio, "wb") as w:
                w.setnchannels(1)
                w.setsampwidth(2)
                w.setframerate(16000)
                w.writeframes(audio_int16(aseed).tobytes())
            res = subprocess.run([sys.executable, script, model, audio], check=True, capture_output=True, text=True)
        ref = json.loads(res.stdout)
        out = {"model_seed": mseed, "audio_seed": aseed, "arch": name, "stages": ref["stages"]}
        with open(os.path.join(args.out, f"logmel_{name}.json"), "w") as f:
            json.dump(out, f, indent=1)
        print(name, "written", list(ref["stages"]))


if __name__ == "__main__":
    main()
