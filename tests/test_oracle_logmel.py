"""The oracle's log-mel front end (oracle/w4j_oracle.c orc_log_mel, restating FeatureExtractor.extract
and padOrTrim with the Java Bluestein FFT) pinned to the reference's own stage-by-stage script
(tools/generate_reference_values.py run on a seeded 30 s WAV and model, via
tests/golden/make_golden_logmel.py).

The script computes the spectrogram with numpy's FFT where the Java code runs a float Bluestein FFT;
the first mel values agree to 1.5e-5 (asserted at 1e-4).  The whole front end plus the oracle's
encoder reproduces the script's encoder output to 2.4e-4 (asserted at 5e-3; the script's exact tanh
GELU against the Java table is the remaining difference).
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml

from .golden.make_golden_logmel import CASES, audio_samples

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module", autouse=True)
def threads():
    O.set_threads(min(16, os.cpu_count() or 1))
    yield
    O.set_threads(1)


def case(name):
    dims, mseed, aseed = CASES[name]
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, mseed, include_encoder=True))
    with open(os.path.join(GOLDEN, f"logmel_{name}.json")) as f:
        return dims, gm, audio_samples(aseed), json.load(f)


def test_log_mel_and_encoder_match_reference_script():
    dims, gm, audio, g = case("mel80_tiny")
    mel = O.log_mel(audio, gm.mel_filters, 2 * dims.n_audio_ctx)
    st = g["stages"]["mel"]
    assert list(mel.shape) == st["shape"]
    np.testing.assert_allclose(mel.ravel()[:8], st["first8"], atol=1e-4)
    xa = O.OracleEncoder(gm).forward(mel)
    np.testing.assert_allclose(xa.ravel()[:8], g["stages"]["encoder_output"]["first8"], atol=5e-3)


def test_log_mel_short_input_and_pad_or_trim():
    """FeatureExtractor.extract pads inputs shorter than n_fft (:75-79); padOrTrim fills the frames past
    the spectrogram's end with its minimum (:137-158)."""
    dims, gm, audio, _ = case("mel80_tiny")
    short = audio[:300]  # fewer samples than n_fft = 400: 3 frames
    mel = O.log_mel(short, gm.mel_filters, 3000)
    assert mel.shape == (dims.n_mels, 3000)
    assert np.all(mel[:, 3:] == mel[:, :3].min())
    assert np.all(mel[:, :3] >= mel[:, :3].min())
    # a longer input is trimmed: the first 3000 of its 3001 frames
    full = O.log_mel(audio, gm.mel_filters, 3001)
    np.testing.assert_array_equal(O.log_mel(audio, gm.mel_filters, 3000), full[:, :3000])
    # the floor: nothing below (max - 8 + 4) / 4
    assert mel.min() >= (mel.max() * 4 - 4 - 8 + 4) / 4 - 1e-6
