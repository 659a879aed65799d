"""w4j_transcribe (WhisperModel.transcribeChunked in the library, the recording resident on the device)
against the oracle's restatement of the same loop (oracle.transcribe_chunked) driven by the GPU's own
per-window stages (encode_audio on the zero-filled 30 s window, decode_with_fallback).  The stages
are deterministic, so the transcript must be identical: same windows, segment times and token ids.
The stages themselves are pinned to the oracle by test_gpu_logmel, test_gpu_encoder and the decoder
tests.
"""
import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200.decoder import WhisperDecoder

from .golden.make_golden_logmel import audio_int16

pytestmark = pytest.mark.gpu

TINY = ggml.ARCHS["tiny.en"]
SOT, EOT, NO_SPEECH, NO_TS, SOT_PREV, TS_BEGIN = [50257, 50258, 50259], 50256, 50361, 50362, 50360, 50363


@pytest.fixture(scope="module")
def dec():
    gm = ggml.parse(ggml.synthetic_model_bytes(TINY, 61, include_encoder=True))
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as d:
        yield d


def reference_loop(dec, audio, ts_begin, condition):
    chunk = 2 * TINY.n_audio_ctx * 160

    def window(a0, n_valid):
        w = np.zeros(chunk, np.float32)
        w[:n_valid] = audio[a0:a0 + n_valid]
        dec.encode_audio(w, slot=0, return_output=False)

    def decode(prompt, max_tokens):
        r = dec.decode_with_fallback_batch([0], [prompt], EOT, max_tokens, suppress_tokens=[EOT],
                                           no_speech_token=NO_SPEECH, timestamp_begin=ts_begin)[0]
        return list(r.tokens), r.avg_logprob, r.no_speech_prob

    return O.transcribe_chunked(audio.size, TINY.n_audio_ctx, TINY.n_text_ctx, SOT, NO_TS, SOT_PREV, ts_begin,
                                condition, window, decode)


@pytest.mark.parametrize("seconds,ts_begin,condition", [(45, -1, True), (10, TS_BEGIN, True), (12, TS_BEGIN, False)])
def test_transcribe_matches_loop_restatement(dec, seconds, ts_begin, condition):
    audio = (audio_int16(70 + seconds, seconds=seconds).astype(np.float32) / 32768.0)
    got, windows = dec.transcribe(audio, SOT, EOT, NO_SPEECH, NO_TS, SOT_PREV, ts_begin=ts_begin, suppress_tokens=[EOT],
                                  condition_on_previous=condition)
    want = reference_loop(dec, audio, ts_begin, condition)
    assert windows >= 1
    assert [(s, e, t) for s, e, t in got] == want
    if ts_begin < 0:
        assert windows == 2  # 45 s: two windows without timestamps


def test_transcribe_empty_audio(dec):
    got, windows = dec.transcribe(np.zeros(0, np.float32), SOT, EOT, NO_SPEECH, NO_TS, SOT_PREV)
    assert got == [] and windows == 0
