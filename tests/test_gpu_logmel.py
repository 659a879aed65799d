"""The log-mel front end on the GPU (w4j_log_mel / w4j_encode_audio, k_logmel.cu) against the oracle's
restatement of FeatureExtractor.extract + padOrTrim and the reference's stage-by-stage script.

The device restates the Java arithmetic operation for operation (float Bluestein FFT with the Java
loop's twiddle recurrence, products and sums without FMA contraction); only log10 (double, then
rounded to float) may round differently in the last place of a double.  So the spectrogram is
compared with the oracle at max-abs 1e-5 and must be bit-identical in at least 99.9 % of its values.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200._lib import IllegalStateError
from whisper4j_b200.decoder import WhisperDecoder

from .golden.make_golden_logmel import CASES, audio_samples

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module", autouse=True)
def threads():
    O.set_threads(min(64, os.cpu_count() or 1))
    yield
    O.set_threads(1)


@pytest.fixture(scope="module")
def tiny():
    dims, mseed, aseed = CASES["mel80_tiny"]
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, mseed, include_encoder=True))
    with open(os.path.join(GOLDEN, "logmel_mel80_tiny.json")) as f:
        g = json.load(f)
    with WhisperDecoder(gm, max_streams=2, max_beam=1) as dec:
        yield dims, gm, audio_samples(aseed), g, dec


def check_mel(got, want):
    assert got.shape == want.shape
    assert np.abs(got - want).max() < 1e-5
    assert np.mean(got == want) >= 0.999


@pytest.mark.parametrize("n", [480000, 160000, 300, 0])
def test_log_mel_matches_oracle(tiny, n):
    dims, gm, audio, _, dec = tiny
    a = audio[:n]
    check_mel(dec.log_mel(a), O.log_mel(a, gm.mel_filters, 2 * dims.n_audio_ctx))


def test_encode_audio_matches_oracle_and_reference(tiny):
    dims, gm, audio, g, dec = tiny
    mel = dec.log_mel(audio)
    np.testing.assert_allclose(mel.ravel()[:8], g["stages"]["mel"]["first8"], atol=1e-4)
    xa = dec.encode_audio(audio, slot=0)
    want = O.OracleEncoder(gm).forward(O.log_mel(audio, gm.mel_filters, 2 * dims.n_audio_ctx))
    assert np.abs(xa - want).max() < 2e-2
    np.testing.assert_allclose(xa.ravel()[:8], g["stages"]["encoder_output"]["first8"], atol=3e-2)
    # the device-set encoder output decodes like the same output passed through the host
    dec.set_encoder_output(xa, slot=1)
    prompt, eot = [50257, 50258, 50259, 50362], 50256
    a = dec.decode_batch([0], [prompt], eot, 8, suppress_tokens=[eot])[0]
    b = dec.decode_batch([1], [prompt], eot, 8, suppress_tokens=[eot])[0]
    assert a.tokens == b.tokens and a.sum_logprob == b.sum_logprob


def test_log_mel_needs_filters():
    dims, mseed, aseed = CASES["mel80_tiny"]
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, mseed, include_encoder=True))
    gm.mel_filters[:] = 0.0  # a file without filters: nothing is uploaded
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as dec:
        with pytest.raises(IllegalStateError):
            dec.log_mel(audio_samples(aseed)[:16000])
