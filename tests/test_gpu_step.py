"""The persistent decode-step kernel (k_step.cu) against the CPU oracle.

With W4J_STEP_KERNEL=1 a decode step of at most eight sequences (streams x beams) after the prompt
runs as ONE kernel: every projection, both attentions, the vocabulary logits and their epilogues,
separated by grid barriers.  These tests run the token loop through it and compare with the oracle
(oracle/w4j_oracle.c, the restatement of WhisperDecoder.java) under the same rules as the chained
kernels: logits within max-abs 2e-2 / relative 1e-2, token ids identical except at a near tie of the
oracle's logits (greedy) or of the beam cut (beam search).  A decode's launch count shows that the
step kernel, not the chain, ran.
"""
import os

import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200.decoder import WhisperDecoder

from .helpers import SMALL, SMALL_OPTS, check_beam, encoder_output, parsed
from .test_gpu_configs import check_greedy, check_score_along, eot_id
from .test_gpu_decoder import check_tokens

pytestmark = pytest.mark.gpu

SO = tuple(sorted(SMALL_OPTS.items()))
TINY = ggml.ARCHS["tiny.en"]


@pytest.fixture(autouse=True, scope="module")
def step_kernel_on():
    old = os.environ.get("W4J_STEP_KERNEL")
    os.environ["W4J_STEP_KERNEL"] = "1"  # read when a decoder context is created
    O.set_threads(min(64, os.cpu_count() or 1))
    yield
    O.set_threads(1)
    if old is None:
        os.environ.pop("W4J_STEP_KERNEL", None)
    else:
        os.environ["W4J_STEP_KERNEL"] = old


def assert_one_kernel_per_step(dec, n_layer):
    """Launches of the last decode: the prompt pass (chained kernels, a few tokens) plus about two per
    step (step kernel, selection); the chained path launches eight or more per layer and step."""
    _, steps, launches = dec.last_timing()
    assert steps > 0 and launches <= 3 * steps + 12 * (8 * n_layer + 4), (steps, launches)


@pytest.fixture(scope="module")
def small():
    gm = parsed(SMALL, 101, "f16", SO)
    d = WhisperDecoder(gm, max_streams=4, max_beam=4)
    o = O.OracleModel(gm)
    xas = [encoder_output(200 + i, SMALL.n_audio_ctx, SMALL.n_text_state) for i in range(4)]
    for i, xa in enumerate(xas):
        d.set_encoder_output(xa, slot=i)
    yield d, o, xas
    d.close()


@pytest.mark.parametrize("slot", [0, 2])
def test_step_greedy_matches_oracle(small, slot):
    dec, ora, xas = small
    prompt = [996, 997, 998, 999]
    r = dec.decode_batch([slot], [prompt], 995, 24, suppress_tokens=[995])[0]
    assert_one_kernel_per_step(dec, SMALL.n_text_layer)
    w = ora.decode(xas[slot], prompt, 995, 24, suppress=[995])
    check_tokens(r.tokens, w["tokens"], ora, xas[slot], prompt)
    if r.tokens == w["tokens"]:
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)


def test_step_greedy_batch_equals_single(small):
    """Every sequence's arithmetic is independent of how many share the step (bit-equal scores)."""
    dec, ora, xas = small
    prompts = [[996, 997, 998, 999], [996, 997, 998, 10], [996, 997, 11, 12]]
    batch = dec.decode_batch([0, 1, 3], prompts, 995, 24, suppress_tokens=[995])
    assert_one_kernel_per_step(dec, SMALL.n_text_layer)
    for (slot, p), rb in zip(zip([0, 1, 3], prompts), batch):
        rs = dec.decode_batch([slot], [p], 995, 24, suppress_tokens=[995])[0]
        assert rb.tokens == rs.tokens
        assert rb.sum_logprob == pytest.approx(rs.sum_logprob, abs=1e-9)
        w = ora.decode(xas[slot], p, 995, 24, suppress=[995])
        check_tokens(rb.tokens, w["tokens"], ora, xas[slot], p)


@pytest.mark.parametrize("beam", [2, 4])
def test_step_beam_matches_oracle(small, beam):
    dec, ora, xas = small
    prompt, eot = [996, 997, 998, 999], 995
    r = dec.decode_beam_batch([1], [prompt], eot, 16, suppress_tokens=[eot], no_speech_token=3, beam_size=beam)[0]
    assert_one_kernel_per_step(dec, SMALL.n_text_layer)
    w = ora.decode_beam(xas[1], prompt, eot, 16, suppress=[eot], no_speech=3, beam=beam, trace=True)
    if check_beam(r.tokens, w, ora, xas[1], prompt, [eot], eot, beam, 16) == "equal":
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)
    assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)


def test_step_beam_two_streams(small):
    """Two streams x four beams: eight sequences, the step kernel's limit."""
    dec, ora, xas = small
    prompts = [[996, 997, 998, 999], [996, 997, 998, 20]]
    got = dec.decode_beam_batch([0, 3], prompts, 995, 10, suppress_tokens=[995], beam_size=4)
    assert_one_kernel_per_step(dec, SMALL.n_text_layer)
    for slot, p, r in zip([0, 3], prompts, got):
        w = ora.decode_beam(xas[slot], p, 995, 10, suppress=[995], beam=4, trace=True)
        check_beam(r.tokens, w, ora, xas[slot], p, [995], 995, 4, 10)


def test_step_tiny_greedy_64_tokens():
    gm = parsed(TINY, 21)
    ora = O.OracleModel(gm)
    xa = encoder_output(22, TINY.n_audio_ctx, TINY.n_text_state)
    prompt, eot = [50257, 50258, 50259, 50362], 50256
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as dec:
        dec.set_encoder_output(xa, 0)
        r = dec.decode(None, prompt, eot, 64, suppress_tokens=[eot])
        assert_one_kernel_per_step(dec, TINY.n_text_layer)
    w = ora.decode(xa, prompt, eot, 64, suppress=[eot])
    check_tokens(r.tokens, w["tokens"], ora, xa, prompt)


def test_step_turbo_batch1_greedy_224_with_timestamps():
    """The north-star latency case (large-v3-turbo, one stream) through the step kernel."""
    dims = ggml.ARCHS["large-v3-turbo"]
    gm = parsed(dims, 1234)
    ora = O.OracleModel(gm)
    xa = encoder_output(7, dims.n_audio_ctx, dims.n_text_state)
    prompt, eot, tsb = [50258, 50259, 50360], eot_id(dims), 50365
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as dec:
        dec.set_encoder_output(xa, 0)
        r = dec.decode(None, prompt, eot, 224, suppress_tokens=[eot], no_speech_token=50363, timestamp_begin=tsb)
        assert_one_kernel_per_step(dec, dims.n_text_layer)
    w = ora.decode(xa, prompt, eot, 224, suppress=[eot], no_speech=50363, ts_begin=tsb)
    assert len(r.tokens) == 224 and r.tokens[0] >= tsb
    if check_greedy(r.tokens, w["tokens"], ora, xa, prompt, [eot], eot, tsb) == "equal":
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2 + 2e-4 * 224)
    check_score_along(r, ora, xa, prompt, [eot], eot, beam_scores=False, ts_begin=tsb)
    assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)
