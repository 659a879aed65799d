"""The audio encoder on the GPU (w4j_encoder_forward: k_encoder.cu + the tensor-core GEMM) against the
oracle's restatement of WhisperEncoder.forward and the reference's own numpy encoder.

Tolerances: the device feeds the attention's q / k / v and probabilities to the tensor cores as f16
(f32 accumulation) and stages the projections' activations as f16 hi / lo pairs; the output is
LayerNorm-ed (unit scale).  Against the oracle (same f16-indexed GELU table as the Java encoder):
max-abs 2e-2.  Against the reference's numpy restatement (exact tanh GELU): max-abs 3e-2.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200._lib import IllegalStateError
from whisper4j_b200.decoder import WhisperDecoder

from .golden.make_golden_encoder import CASES, mel_input
from .helpers import SMALL, SMALL_OPTS, parsed

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ATOL_ORACLE, ATOL_GOLDEN = 2e-2, 3e-2


@pytest.fixture(scope="module", autouse=True)
def threads():
    O.set_threads(min(64, os.cpu_count() or 1))
    yield
    O.set_threads(1)


def encoder_case(name):
    dims, mseed, xseed, opts, _ = CASES[name]
    gm = ggml.parse(ggml.synthetic_model_bytes(dims, mseed, include_encoder=True, **opts))
    return dims, gm, mel_input(xseed, dims.n_mels, 2 * dims.n_audio_ctx)


@pytest.mark.parametrize("name", ["enc_small", "enc_tiny"])
def test_encoder_matches_oracle_and_reference(name):
    dims, gm, mel = encoder_case(name)
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as dec:
        got = dec.encode(mel)
        again = dec.encode(mel)
    assert got.shape == (dims.n_audio_ctx, dims.n_audio_state) and np.isfinite(got).all()
    np.testing.assert_array_equal(got, again)  # deterministic
    want = O.OracleEncoder(gm).forward(mel)
    err = np.abs(got - want).max()
    assert err < ATOL_ORACLE, f"max-abs {err} against the oracle"
    with open(os.path.join(GOLDEN, f"encoder_{name}.json")) as f:
        g = json.load(f)
    rows = sorted(int(r) for r in g["rows"])
    ref = np.array([g["rows"][str(r)] for r in rows], np.float32)
    assert np.abs(got[rows] - ref).max() < ATOL_GOLDEN


def test_encoder_output_feeds_the_decoder_on_device():
    """encode(mel, slot) sets the stream's cross K/V on the device; decoding from it equals decoding
    from the same encoder output passed through the host."""
    dims, gm, mel = encoder_case("enc_small")
    prompt, eot = [996, 997, 998, 999], 995
    with WhisperDecoder(gm, max_streams=2, max_beam=1) as dec:
        xa = dec.encode(mel, slot=0)
        dec.set_encoder_output(xa, slot=1)
        a = dec.decode_batch([0], [prompt], eot, 12, suppress_tokens=[eot])[0]
        b = dec.decode_batch([1], [prompt], eot, 12, suppress_tokens=[eot])[0]
    assert a.tokens == b.tokens and a.sum_logprob == b.sum_logprob
    ora = O.OracleModel(gm)
    w = ora.decode(O.OracleEncoder(gm).forward(mel), prompt, eot, 12, suppress=[eot])
    assert len(a.tokens) == 12 and len(w["tokens"]) == 12


def test_encoder_errors():
    dims, gm, mel = encoder_case("enc_small")
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as dec:
        with pytest.raises(ValueError):
            dec.encode(mel[:, :-2])  # frames must be 2 n_audio_ctx
        with pytest.raises(ValueError):
            dec.encode(mel, slot=5)  # slot out of range
    # a model without encoder tensors: the decoder loads, the encoder reports what is missing
    with WhisperDecoder(parsed(SMALL, 101, "f16", tuple(sorted(SMALL_OPTS.items()))), max_streams=1, max_beam=1) as dec:
        with pytest.raises(IllegalStateError):
            dec.encode(np.zeros((SMALL.n_mels, 2 * SMALL.n_audio_ctx), np.float32))
