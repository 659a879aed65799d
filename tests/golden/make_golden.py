#!/usr/bin/env python3
"""Generate golden decode-step vectors from the reference's own Python restatement.

Run where a checkout of the reference is available; its path is given with
--reference.  It imports the reference's
``tools/validate_decode_steps.py`` (``load_ggml`` and ``decoder_step``, the
numpy restatement that the reference's ValidateAgainstReferenceTest pins the
Java decoder against), feeds it a seeded synthetic GGML model written by
``whisper4j_b200.ggml`` and a seeded encoder output, and records per greedy step
the chosen token, the top-5 ids and values and the first 8 logits — the same
quantities ValidateAgainstReferenceTest.java:145-161 and :173-255 compare.

The fixtures are small JSON files; the model weights and encoder output are
regenerated from their seeds by the tests.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from whisper4j_b200 import ggml  # noqa: E402

# name -> (dims, model seed, xa seed, extra synthetic options, prompt, steps)
CASES = {
    "small_rand": (ggml.ModelDimensions(80, 96, 128, 2, 1, 1000, 64, 128, 2, 2), 11, 12,
                   dict(bias_std=0.02, ln_std=0.1, std=0.05), [996, 997, 998, 999], 12),
    "tiny_en": (ggml.ARCHS["tiny.en"], 21, 22, dict(), [50257, 50258, 50259, 50362], 10),
}


def encoder_output(seed: int, n_audio_ctx: int, d: int) -> np.ndarray:
    """Seeded stand-in for the encoder output: rows standardised like ln_post output (gamma=1, beta=0)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n_audio_ctx, d), dtype=np.float32)
    x = (x - x.mean(axis=1, keepdims=True)) / x.std(axis=1, keepdims=True)
    return x.astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of sparrowlogic/whisper4j (its tools/ directory)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "tools"))
    import validate_decode_steps as ref  # the reference's numpy restatement

    for name, (dims, mseed, xseed, opts, prompt, n_steps) in CASES.items():
        buf = ggml.synthetic_model_bytes(dims, mseed, **opts)
        with tempfile.NamedTemporaryFile(suffix=".bin", delete=False) as f:
            f.write(buf)
            path = f.name
        try:
            W, hp, _ = ref.load_ggml(path)
        finally:
            os.unlink(path)
        xa = encoder_output(xseed, dims.n_audio_ctx, dims.n_text_state)[None]
        kv = {}
        cur, offset, steps = list(prompt), 0, []
        for step in range(n_steps):
            logits = ref.decoder_step(cur, xa, W, hp, kv, offset)
            last = logits[0, -1].astype(np.float32)
            tok = int(np.argmax(last))
            order = np.argsort(-last, kind="stable")[:5]
            steps.append({
                "step": step, "input": [int(t) for t in cur], "token": tok,
                "top5": [int(i) for i in order], "top5_scores": [float(last[i]) for i in order],
                "first8": [float(v) for v in last[:8]],
                "row0_first8": [float(v) for v in logits[0, 0, :8].astype(np.float32)],
                "mean": float(last.mean()), "std": float(last.std()),
            })
            offset += len(cur)
            cur = [tok]
        out = {"case": name, "dims": dims.__dict__ if hasattr(dims, "__dict__") else None,
               "model_seed": mseed, "xa_seed": xseed, "synthetic_options": opts, "prompt": prompt,
               "generator": "reference tools/validate_decode_steps.py (load_ggml, decoder_step)",
               "steps": steps}
        out["dims"] = {k: getattr(dims, k) for k in dims.__dataclass_fields__}
        with open(os.path.join(args.out, f"decode_steps_{name}.json"), "w") as f:
            json.dump(out, f, indent=1)
        print(name, [s["token"] for s in steps])


if __name__ == "__main__":
    main()
