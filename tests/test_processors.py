"""Logit processors and host policy against hand-derived answers from the reference's Java.

n-gram block: WhisperDecoder.java:472-476, :543-564; timestamp rules :484-541;
compression ratio :628-647 with WhisperDecoderTest.java's cases; needsFallback :435-440.
The processors are checked in the oracle here (CPU); the device copies are compared with
the oracle through full decodes in the GPU tests.
"""
import zlib

import numpy as np
import pytest

from oracle import oracle as O

NEG = -np.inf


def blocked(out):
    return sorted(np.nonzero(np.isneginf(out))[0].tolist())


def test_ngram_trigram_block():
    # generated = a b c a b -> suffix (a, b) matched at i=0 -> block c
    out = O.apply_repetition_penalty(np.zeros(10), [1, 2, 3, 1, 2])
    assert blocked(out) == [3]


def test_ngram_four_gram_block():
    # 5 6 7 8 5 6 7 -> 3-gram suffix (6,7) -> block 8; 4-gram suffix (5,6,7) -> block 8
    out = O.apply_repetition_penalty(np.zeros(10), [5, 6, 7, 8, 5, 6, 7])
    assert blocked(out) == [8]


def test_ngram_short_history():
    assert blocked(O.apply_repetition_penalty(np.zeros(10), [])) == []
    assert blocked(O.apply_repetition_penalty(np.zeros(10), [4, 4])) == []
    assert blocked(O.apply_repetition_penalty(np.zeros(10), [4, 4, 4])) == [4]


def test_timestamp_first_step():
    V, tb, eot = 200, 100, 90
    out = O.apply_timestamp_rules(np.zeros(V), [], tb, eot, True)
    # <|notimestamps|> (tb-1), every text token, and timestamps past tb+50
    assert blocked(out) == list(range(0, tb)) + list(range(tb + 51, V))


def test_timestamp_pair_rules():
    V, tb, eot = 200, 100, 90
    # last two are timestamps -> text must follow (block all timestamps); non-decreasing: block [tb, last)
    out = O.apply_timestamp_rules(np.zeros(V), [5, 110, 120], tb, eot, False)
    assert blocked(out) == [tb - 1] + list(range(tb, V))
    # single timestamp after text -> only timestamps or eot; block < eot and [tb, last+1)
    out = O.apply_timestamp_rules(np.zeros(V), [5, 6, 120], tb, eot, False)
    assert blocked(out) == list(range(0, eot)) + [tb - 1] + list(range(tb, 121))
    # text after a timestamp: block [tb, last_ts)
    out = O.apply_timestamp_rules(np.zeros(V), [104, 5, 6], tb, eot, False)
    assert blocked(out) == [tb - 1] + list(range(tb, 104))


def java_ratio(tokens):
    b = bytearray()
    for t in tokens:
        b += bytes([t & 0xFF, (t >> 8) & 0xFF])
    return len(b) / max(1, len(zlib.compress(bytes(b), 6))) if tokens else 0.0


def test_compression_ratio_matches_zlib():
    from whisper4j_b200.decoder import compression_ratio
    assert compression_ratio([]) == 0.0  # WhisperDecoderTest.java:8-11
    rep = [42] * 100
    assert compression_ratio(rep) > 2.0  # :13-22
    rnd = [i * 137 % 50000 for i in range(100)]
    assert compression_ratio(rnd) < 2.5  # :24-33
    for toks in (rep, rnd, [1, 2, 3], list(range(300))):
        assert compression_ratio(toks) == pytest.approx(java_ratio(toks), rel=1e-6)


@pytest.mark.parametrize("cr,avg,nsp,want", [
    (2.5, -0.5, 0.1, True),    # too repetitive
    (2.5, -1.5, 0.7, False),   # repetitive but silence
    (1.5, -1.5, 0.1, True),    # low confidence
    (1.5, -1.5, 0.7, False),   # low confidence but silence
    (1.5, -0.5, 0.1, False),
])
def test_needs_fallback(cr, avg, nsp, want):
    from whisper4j_b200.decoder import needs_fallback
    assert needs_fallback(cr, avg, nsp) is want
