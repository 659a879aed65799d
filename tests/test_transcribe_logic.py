"""The oracle's restatement of WhisperModel.transcribeChunked's segment, prompt and seek logic
(oracle/oracle.py, WhisperModel.java:334-530) on hand-derived cases read off the Java code."""
import numpy as np

from oracle import oracle as O

TS = 50364  # a timestamp_begin id; only the comparison t >= TS matters


def test_segments_split_at_consecutive_timestamps():
    # ts positions 0, 3, 4, 6: only (3, 4) is consecutive -> one slice [0, 4); the tail after the last
    # consecutive pair is not emitted (:458-489)
    got = O.timestamp_segments([TS, 10, 11, TS + 50, TS + 50, 12, TS + 80], TS, 0.0, 0.02)
    assert got == [(0.0, O.f32(np.float32(50) * np.float32(0.02)), [10, 11])]
    # a slice without text is dropped, the next one starts after it
    got = O.timestamp_segments([TS, TS, 7, TS + 4, TS + 4], TS, 1.5, 0.02)
    assert got == [(1.5, O.f32(np.float32(1.5) + np.float32(4) * np.float32(0.02)), [7])]


def test_segments_with_fewer_than_two_timestamps():
    # one timestamp: the segment ends at it (:444-456); none: 30 s after the window start
    assert O.timestamp_segments([TS + 10, 5, 6], TS, 0.0, 0.02) == [(0.0, O.f32(np.float32(10) * np.float32(0.02)), [5, 6])]
    assert O.timestamp_segments([5, 6], TS, 2.0, 0.02) == [(2.0, 32.0, [5, 6])]
    assert O.timestamp_segments([TS + 3], TS, 0.0, 0.02) == []


def test_prompt_with_context():
    base, prev = [1, 2, 3], [9, 8, 7, 6]
    assert O.prompt_with_context(base, prev, 99, 10, True) == base  # no room (:515-517)
    assert O.prompt_with_context(base, prev, 99, 20, True) == [99, 9, 8, 7, 6, 1, 2, 3]
    assert O.prompt_with_context(base, prev, 99, 14, True) == [99, 7, 6, 1, 2, 3]  # the last tokens kept
    assert O.prompt_with_context(base, prev, 99, 20, False) == base
    assert O.prompt_with_context(base, [], 99, 20, True) == base


def test_seek_advances_from_the_last_timestamp():
    windows, prompts = [], []

    def window(a0, n_valid):
        windows.append((a0, n_valid))

    answers = iter([
        ([TS, 5, 6, TS + 1000, TS + 1000, 7, TS + 1000], -0.5, 0.1),  # last timestamp 20 s: seek += 2000
        ([8, 9], -0.3, 0.1),                                          # no timestamp: seek += the window
    ])

    def decode(prompt, max_tokens):
        prompts.append((list(prompt), max_tokens))
        return next(answers)

    segs = O.transcribe_chunked(16000 * 45, 1500, 448, [50258, 50259, 50360], 50364, 50362, TS, True, window, decode)
    assert windows == [(0, 480000), (320000, 400000)]
    assert prompts[0] == ([50258, 50259, 50360], 224)
    # the second window conditions on the first's tokens and decodes at most 224 * 2500 / 3000 tokens
    assert prompts[1][0][0] == 50362 and prompts[1][0][-3:] == [50258, 50259, 50360] and prompts[1][1] == 186
    assert segs[0] == (0.0, 20.0, [5, 6])
    assert segs[1][2] == [8, 9] and segs[1][0] == O.f32(np.float32(2000) * np.float32(160.0) / np.float32(16000.0))


def test_no_speech_and_hallucination_retry():
    calls = []

    def decode(prompt, max_tokens):
        calls.append(list(prompt))
        if len(calls) == 1:
            return [5, 6], -0.2, 0.1            # window 1: fine, becomes the context
        if len(calls) == 2:
            return [7], -1.5, 0.1               # window 2 with context: too unlikely -> retried without
        if len(calls) == 3:
            return [8], -1.2, 0.9               # the retry: no speech -> skipped
        return [9], -0.1, 0.0

    segs = O.transcribe_chunked(16000 * 75, 1500, 448, [1, 2], 3, 4, -1, True, lambda a, n: None, decode)
    assert calls[1][0] == 4 and calls[2] == [1, 2, 3]   # retry uses the plain prompt (no context)
    assert calls[3] == [1, 2, 3]                         # the context was reset by the retry
    assert [s[2] for s in segs] == [[5, 6], [9]]
