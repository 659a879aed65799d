"""Batched decoding against the CPU oracle: with 16 or more live sequences every projection of
the decode step runs on the tcgen05 kernel (LayerNorm prologue, token + position embedding of
layer 0, Q/K/V with the self-cache scatter, residual and GELU epilogues), and with many
(stream, head) pairs cross-attention runs on the streaming kernel.

WhisperDecoder.decode / decodeBeam (WhisperDecoder.java) per stream; tolerances as in the
single-stream decoder tests: identical ids except at near ties of the oracle's logits.
"""
import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200.decoder import WhisperDecoder

from .helpers import SMALL, SMALL_OPTS, check_beam, encoder_output, parsed
from .test_gpu_decoder import check_tokens

pytestmark = pytest.mark.gpu

SO = tuple(sorted(SMALL_OPTS.items()))
TINY = ggml.ARCHS["tiny.en"]
N_STREAMS = 20


@pytest.fixture(scope="module")
def wide():
    gm = parsed(SMALL, 101, "f16", SO)
    d = WhisperDecoder(gm, max_streams=N_STREAMS, max_beam=2)
    o = O.OracleModel(gm)
    xas = [encoder_output(300 + i, SMALL.n_audio_ctx, SMALL.n_text_state) for i in range(N_STREAMS)]
    for i, xa in enumerate(xas):
        d.set_encoder_output(xa, slot=i)
    yield d, o, xas
    d.close()


def _prompts(n):
    return [[996, 997, 998, 10 + i] for i in range(n)]


def test_greedy_20_streams_match_oracle(wide):
    dec, ora, xas = wide
    slots = list(range(N_STREAMS))
    prompts = _prompts(N_STREAMS)
    res = dec.decode_batch(slots, prompts, 995, 24, suppress_tokens=[995], no_speech_token=3)
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode(xas[s], p, 995, 24, suppress=[995], no_speech=3)
        check_tokens(r.tokens, w["tokens"], ora, xas[s], p)
        if r.tokens == w["tokens"]:
            assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2 + 1e-3 * abs(w["sum_logprob"]))
        assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)


def test_greedy_16_streams_with_eot(wide):
    """Sequences finish at different steps: finished rows leave the projections' epilogues."""
    dec, ora, xas = wide
    slots = list(range(16))
    prompts = _prompts(16)
    free = ora.decode(xas[0], prompts[0], 995, 16, suppress=[995])
    eot = free["tokens"][3]
    res = dec.decode_batch(slots, prompts, eot, 16)
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode(xas[s], p, eot, 16)
        check_tokens(r.tokens, w["tokens"], ora, xas[s], p)


def test_beam_2_times_10_streams_match_oracle(wide):
    dec, ora, xas = wide
    slots = list(range(10))
    prompts = _prompts(10)
    res = dec.decode_beam_batch(slots, prompts, 995, 12, suppress_tokens=[995], beam_size=2)
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode_beam(xas[s], p, 995, 12, suppress=[995], beam=2, trace=True)
        if check_beam(r.tokens, w, ora, xas[s], p, [995], 995, 2, 12) == "equal":
            assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)
        assert len(r.tokens) == 12


# ---------------------------------------------------------------------------
# more than 32 live rows: the tcgen05 vocabulary pass runs once per chunk of at most 32 rows
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def wide40():
    gm = parsed(SMALL, 101, "f16", SO)
    d = WhisperDecoder(gm, max_streams=40, max_beam=4)
    o = O.OracleModel(gm)
    xas = [encoder_output(500 + i, SMALL.n_audio_ctx, SMALL.n_text_state) for i in range(40)]
    for i, xa in enumerate(xas):
        d.set_encoder_output(xa, slot=i)
    yield d, o, xas
    d.close()


def test_greedy_40_streams_match_oracle(wide40):
    dec, ora, xas = wide40
    slots = list(range(40))
    prompts = [[996, 997, 998, 10 + i] for i in range(40)]
    res = dec.decode_batch(slots, prompts, 995, 16, suppress_tokens=[995], no_speech_token=3)
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode(xas[s], p, 995, 16, suppress=[995], no_speech=3)
        check_tokens(r.tokens, w["tokens"], ora, xas[s], p)
        if r.tokens == w["tokens"]:
            assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2 + 1e-3 * abs(w["sum_logprob"]))
        assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)


def test_beam_4_times_10_streams_match_oracle(wide40):
    dec, ora, xas = wide40
    slots = list(range(10))
    prompts = [[996, 997, 998, 10 + i] for i in range(10)]
    res = dec.decode_beam_batch(slots, prompts, 995, 10, suppress_tokens=[995], beam_size=4)
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode_beam(xas[s], p, 995, 10, suppress=[995], beam=4, trace=True)
        if check_beam(r.tokens, w, ora, xas[s], p, [995], 995, 4, 10) == "equal":
            assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)
        assert len(r.tokens) == 10


# ---------------------------------------------------------------------------
# tiny.en (6 heads, 1500 encoder rows) with 8 streams: more (group, head, split) work than one
# wave of the cluster attention kernel, so cross-attention runs on the streaming kernel
# (persistent blocks, per-split partials in global memory, last-arriver combine)
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def tiny8():
    gm = parsed(TINY, 31)
    d = WhisperDecoder(gm, max_streams=8, max_beam=2)
    o = O.OracleModel(gm)
    xas = [encoder_output(400 + i, TINY.n_audio_ctx, TINY.n_text_state) for i in range(8)]
    for i, xa in enumerate(xas):
        d.set_encoder_output(xa, slot=i)
    yield d, o, xas
    d.close()


def _tiny_prompts(n):
    return [[50257, 50258, 50259, 300 + 7 * i] for i in range(n)]


def test_tiny_greedy_8_streams_match_oracle(tiny8):
    dec, ora, xas = tiny8
    slots, prompts = list(range(8)), _tiny_prompts(8)
    res = dec.decode_batch(slots, prompts, 50256, 12, suppress_tokens=[50256])
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode(xas[s], p, 50256, 12, suppress=[50256])
        check_tokens(r.tokens, w["tokens"], ora, xas[s], p)
        if r.tokens == w["tokens"]:
            assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2 + 1e-3 * abs(w["sum_logprob"]))


def test_tiny_beam_2_times_8_streams_match_oracle(tiny8):
    dec, ora, xas = tiny8
    slots, prompts = list(range(8)), _tiny_prompts(8)
    res = dec.decode_beam_batch(slots, prompts, 50256, 8, suppress_tokens=[50256], beam_size=2)
    for s, p, r in zip(slots, prompts, res):
        w = ora.decode_beam(xas[s], p, 50256, 8, suppress=[50256], beam=2, trace=True)
        if check_beam(r.tokens, w, ora, xas[s], p, [50256], 50256, 2, 8) == "equal":
            assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)
        assert len(r.tokens) == 8


# 129 .. 256 live rows: the vocabulary pass is one launch over two 128-row chunks of staged rows
# (k_logits_big), one record per (row, 128-row embedding tile) merged by the select kernel.
N_BIG = 136


@pytest.fixture(scope="module")
def wide136():
    gm = parsed(SMALL, 103, "f16", SO)
    xas = [encoder_output(700 + i, SMALL.n_audio_ctx, SMALL.n_text_state) for i in range(N_BIG)]
    yield gm, O.OracleModel(gm), xas


def _decode_all(gm, xas, env, monkeypatch):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    with WhisperDecoder(gm, max_streams=N_BIG, max_beam=1) as d:
        for i, xa in enumerate(xas):
            d.set_encoder_output(xa, slot=i)
        prompts = [[996, 997, 998, 10 + i % 900] for i in range(N_BIG)]
        return prompts, d.decode_batch(list(range(N_BIG)), prompts, 995, 12, suppress_tokens=[995], no_speech_token=3)


def test_greedy_136_streams_one_launch_vocabulary(wide136, monkeypatch):
    gm, ora, xas = wide136
    prompts, res = _decode_all(gm, xas, {}, monkeypatch)
    for s in range(0, N_BIG, 9):  # a sample of the streams against the oracle
        w = ora.decode(xas[s], prompts[s], 995, 12, suppress=[995], no_speech=3)
        check_tokens(res[s].tokens, w["tokens"], ora, xas[s], prompts[s])
        if res[s].tokens == w["tokens"]:
            assert res[s].sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2 + 1e-3 * abs(w["sum_logprob"]))
        assert res[s].no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)
    # the same decode with 32-row vocabulary launches (one record per block): same decisions
    _, ref = _decode_all(gm, xas, {"W4J_LOGITS_CHUNKED": "1"}, monkeypatch)
    same = [a.tokens == b.tokens for a, b in zip(res, ref)]
    assert sum(same) >= 0.95 * N_BIG
    for a, b, eq in zip(res, ref, same):
        if eq:
            assert a.sum_logprob == pytest.approx(b.sum_logprob, abs=1e-3)
            assert a.no_speech_prob == pytest.approx(b.no_speech_prob, rel=1e-3, abs=1e-7)
