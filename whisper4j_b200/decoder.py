"""Host-side mirror of the reference's ``WhisperDecoder`` over libwhisper4j_cuda.

Same operations, argument meanings and error behaviour as
com.sparrowlogic.whisper4j.nn.WhisperDecoder (nn/WhisperDecoder.java):

    WhisperDecoder(weights, dims)                 ctor          :36-56
    forward(tokens, xa, kv_cache)                 forward       :59-104
    decode(xa, prompt, eot, max_tokens, ...)      decode        :151-204
    decode_beam(...)                              decodeBeam    :214-394
    decode_with_fallback(...)                     decodeWithFallback :110-149
    DecodeResult                                  record        :672-673
    compression_ratio(tokens)                     compressionRatio :628-647

IllegalArgumentException maps to ValueError and IllegalStateException to
IllegalStateError.  Beyond the reference, the ``*_batch`` methods decode many
independent streams (audio chunks) in one device loop.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple, Sequence

import numpy as np

from . import ggml
from ._lib import Dims, Result, Segment, TranscribeOpts, Transcript, check, lib


class DecodeResult(NamedTuple):
    tokens: list
    avg_logprob: float
    compression_ratio: float
    no_speech_prob: float
    temperature: float
    sum_logprob: float = 0.0


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def compression_ratio(tokens: Sequence[int]) -> float:
    t = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.int32))
    return float(lib().w4j_compression_ratio(_ptr(t) if t.size else None, int(t.size)))


def needs_fallback(compression: float, avg_logprob: float, no_speech_prob: float) -> bool:
    return bool(lib().w4j_needs_fallback(compression, avg_logprob, no_speech_prob))


class KvCache:
    """A stream's self-attention cache on the device (the reference's kvCache map)."""

    def __init__(self, decoder: "WhisperDecoder", slot: int):
        self.decoder = decoder
        self.slot = slot

    def reset(self):
        check(lib().w4j_reset_cache(self.decoder._ctx, self.slot))


class WhisperDecoder:
    """Decoder on one GPU, built from a parsed GGML model (whisper4j_b200.ggml.GgmlModel)."""

    def __init__(self, model, dims: ggml.ModelDimensions | None = None, device: int = 0, max_streams: int = 1,
                 max_beam: int = 5):
        if isinstance(model, str):
            model = ggml.load(model)
        elif isinstance(model, (bytes, bytearray, memoryview)):
            model = ggml.parse(model)
        self.model = model
        self.dims = dims or model.dims
        dm = self.dims
        self.max_streams, self.max_beam = max_streams, max_beam
        cd = Dims(dm.n_mels, dm.n_audio_ctx, dm.n_audio_state, dm.n_audio_head, dm.n_audio_layer,
                  dm.n_vocab, dm.n_text_ctx, dm.n_text_state, dm.n_text_head, dm.n_text_layer)
        h = ctypes.c_void_p()
        check(lib().w4j_ctx_create(ctypes.byref(cd), device, max_streams, max_beam, ctypes.byref(h)))
        self._ctx = h
        try:
            for name, t in model.tensors.items():
                if not name.startswith(("decoder.", "encoder.")):
                    continue
                ne = (ctypes.c_int64 * len(t.ne))(*t.ne)
                buf = np.frombuffer(t.data, dtype=np.uint8)
                check(lib().w4j_upload_tensor(self._ctx, name.encode(), t.ttype, ne, len(t.ne), _ptr(buf), buf.size))
            check(lib().w4j_finalize(self._ctx))
            mf = getattr(model, "mel_filters", None)
            if mf is not None and mf.ndim == 2 and mf.shape[0] == dm.n_mels and 2 <= mf.shape[1] <= 257 and mf.any():
                f = np.ascontiguousarray(mf, dtype=np.float32)
                check(lib().w4j_upload_mel_filters(self._ctx, _ptr(f), f.shape[0], f.shape[1]))
        except Exception:
            self.close()
            raise
        self._xa_ids = {}

    # -- lifecycle -------------------------------------------------------------
    def close(self):
        if getattr(self, "_ctx", None):
            lib().w4j_ctx_destroy(self._ctx)
            self._ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- inputs ------------------------------------------------------------------
    def set_encoder_output(self, xa, slot: int = 0):
        """Store stream ``slot``'s encoder output (n_audio_ctx x n_audio_state) and project cross K/V."""
        if hasattr(xa, "is_cuda") and xa.is_cuda:
            t = xa.contiguous().float()
            check(lib().w4j_set_encoder_output_device(self._ctx, slot, ctypes.c_void_p(t.data_ptr()), t.shape[-2]))
        else:
            a = np.ascontiguousarray(np.asarray(xa, dtype=np.float32).reshape(-1, self.dims.n_text_state))
            check(lib().w4j_set_encoder_output(self._ctx, slot, _ptr(a), a.shape[0]))
        self._xa_ids[slot] = id(xa)

    def encode(self, mel, slot: int | None = None, return_output: bool = True):
        """WhisperEncoder.forward on the device: mel (n_mels x 2 n_audio_ctx, as the reference's
        (1, n_mels, n_ctx) input) -> encoder output xa (n_audio_ctx x n_audio_state), with the model's
        "encoder.*" weights on this decoder's device.  With ``slot`` the output also becomes that
        stream's encoder output (cross K/V projected on the device, no host round trip)."""
        dm = self.dims
        m = np.ascontiguousarray(np.asarray(mel, dtype=np.float32))
        if m.ndim == 3 and m.shape[0] == 1:
            m = m[0]
        if m.ndim != 2 or m.shape[0] != dm.n_mels:
            raise ValueError(f"mel must be ({dm.n_mels}, {2 * dm.n_audio_ctx}), got {m.shape}")
        out = np.empty((dm.n_audio_ctx, dm.n_audio_state), np.float32) if return_output else None
        check(lib().w4j_encoder_forward(self._ctx, _ptr(m), m.shape[1], _ptr(out) if out is not None else None,
                                        -1 if slot is None else slot))
        if slot is not None:
            self._xa_ids[slot] = ("encoder", id(mel))
        return out

    def log_mel(self, audio) -> np.ndarray:
        """FeatureExtractor.extract + padOrTrim on the device: 16 kHz mono samples -> the
        (n_mels, 2 n_audio_ctx) log-mel spectrogram, with the model file's mel filters."""
        a = np.ascontiguousarray(np.asarray(audio, dtype=np.float32).reshape(-1))
        out = np.empty((self.dims.n_mels, 2 * self.dims.n_audio_ctx), np.float32)
        check(lib().w4j_log_mel(self._ctx, _ptr(a) if a.size else None, a.size, _ptr(out)))
        return out

    def encode_audio(self, audio, slot: int | None = None, return_output: bool = True):
        """One chunk's front end on the device: log-mel, encoder, and with ``slot`` that stream's
        cross K/V (WhisperModel.transcribe's feature + encoder stage)."""
        a = np.ascontiguousarray(np.asarray(audio, dtype=np.float32).reshape(-1))
        dm = self.dims
        out = np.empty((dm.n_audio_ctx, dm.n_audio_state), np.float32) if return_output else None
        check(lib().w4j_encode_audio(self._ctx, _ptr(a) if a.size else None, a.size,
                                     _ptr(out) if out is not None else None, -1 if slot is None else slot))
        if slot is not None:
            self._xa_ids[slot] = ("audio", id(audio))
        return out

    def transcribe(self, audio, sot, eot, no_speech, no_timestamps, sot_prev, ts_begin=-1, suppress_tokens=(),
                   beam_size=1, condition_on_previous=True, seed=0):
        """WhisperModel.transcribeChunked on the device (stream 0 is the working stream): 30 s windows
        from the seek position through log-mel, encoder and decodeWithFallback, cut into segments.
        Returns (segments, windows) with segments [(start_s, end_s, token_ids)]."""
        a = np.ascontiguousarray(np.asarray(audio, dtype=np.float32).reshape(-1))
        sot_a = np.ascontiguousarray(sot, dtype=np.int32)
        sup = np.ascontiguousarray(list(suppress_tokens) or [0], dtype=np.int32)
        i32p = ctypes.POINTER(ctypes.c_int32)
        o = TranscribeOpts(sot_a.ctypes.data_as(i32p), sot_a.size, eot, no_speech, no_timestamps, sot_prev, ts_begin,
                           sup.ctypes.data_as(i32p), len(suppress_tokens), beam_size, int(condition_on_previous), seed)
        # the seek advances at least 2 frames (20 ms) per window: every window's tokens fit this bound
        windows = a.size // 320 + 2
        cap_tok = windows * (self.dims.n_text_ctx // 2) + 16
        toks = np.zeros(cap_tok, np.int32)
        segs = (Segment * cap_tok)()
        t = Transcript(toks.ctypes.data_as(i32p), cap_tok, segs, cap_tok, 0, 0, 0)
        check(lib().w4j_transcribe(self._ctx, _ptr(a) if a.size else None, a.size, ctypes.byref(o), ctypes.byref(t)))
        out = [(segs[i].start, segs[i].end, toks[segs[i].token_begin:segs[i].token_begin + segs[i].n_tokens].tolist())
               for i in range(t.n_segments)]
        self._xa_ids.pop(0, None)
        return out, t.n_windows

    def _slot_for(self, xa, slot):
        if xa is None:
            return slot
        if self._xa_ids.get(slot) != id(xa):
            self.set_encoder_output(xa, slot)
        return slot

    def new_cache(self, slot: int = 0) -> KvCache:
        c = KvCache(self, slot)
        c.reset()
        return c

    # -- WhisperDecoder.forward ---------------------------------------------------
    def forward(self, tokens: Sequence[int], xa=None, kv_cache: KvCache | None = None, slot: int = 0) -> np.ndarray:
        """Logits (len(tokens), n_vocab) as float32; ``kv_cache`` None runs without a cache."""
        if kv_cache is not None:
            slot = kv_cache.slot
        slot = self._slot_for(xa, slot)
        tok = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.int32))
        out = np.empty((tok.size, self.dims.n_vocab), dtype=np.float32)
        check(lib().w4j_forward(self._ctx, slot, _ptr(tok) if tok.size else None, int(tok.size),
                                1 if kv_cache is not None else 0, _ptr(out)))
        return out

    # -- decode loops ---------------------------------------------------------------
    def _result_buffers(self, n, max_tokens):
        toks = np.zeros((n, max(max_tokens, 1)), np.int32)
        lens = np.zeros(n, np.int32)
        sums = np.zeros(n, np.float64)
        avgs = np.zeros(n, np.float32)
        crs = np.zeros(n, np.float32)
        nsp = np.zeros(n, np.float32)
        r = Result(toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                   sums.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), avgs.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                   crs.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), nsp.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return r, (toks, lens, sums, avgs, crs, nsp)

    @staticmethod
    def _collect(bufs, temps):
        toks, lens, sums, avgs, crs, nsp = bufs
        return [DecodeResult(toks[i, :lens[i]].tolist(), float(avgs[i]), float(crs[i]), float(nsp[i]),
                             float(temps[i]), float(sums[i])) for i in range(len(lens))]

    @staticmethod
    def _prompts(prompts):
        p = np.ascontiguousarray(np.asarray(prompts, dtype=np.int32))
        if p.ndim != 2 or p.shape[1] < 1:
            raise ValueError("prompts must be a non-empty (n_streams, n_prompt) array")
        return p

    @staticmethod
    def _suppress(suppress):
        s = np.ascontiguousarray(np.asarray(list(suppress) if suppress is not None else [], dtype=np.int32))
        return s, (_ptr(s) if s.size else None)

    def decode_batch(self, slots, prompts, eot, max_tokens, suppress_tokens=(), no_speech_token=-1,
                     temperature=0.0, timestamp_begin=-1, seed=0):
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        pr = self._prompts(prompts)
        sp, spp = self._suppress(suppress_tokens)
        r, bufs = self._result_buffers(sl.size, max_tokens)
        check(lib().w4j_decode(self._ctx, _ptr(sl), sl.size, _ptr(pr), pr.shape[1], eot, max_tokens, spp, sp.size,
                               no_speech_token, float(temperature), timestamp_begin, seed, ctypes.byref(r)))
        return self._collect(bufs, [temperature] * sl.size)

    def decode_beam_batch(self, slots, prompts, eot, max_tokens, suppress_tokens=(), no_speech_token=-1,
                          timestamp_begin=-1, beam_size=5):
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        pr = self._prompts(prompts)
        sp, spp = self._suppress(suppress_tokens)
        r, bufs = self._result_buffers(sl.size, max_tokens)
        check(lib().w4j_decode_beam(self._ctx, _ptr(sl), sl.size, _ptr(pr), pr.shape[1], eot, max_tokens, spp,
                                    sp.size, no_speech_token, timestamp_begin, beam_size, ctypes.byref(r)))
        return self._collect(bufs, [0.0] * sl.size)

    def decode_with_fallback_batch(self, slots, prompts, eot, max_tokens, suppress_tokens=(), no_speech_token=-1,
                                   timestamp_begin=-1, beam_size=1, seed=0):
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        pr = self._prompts(prompts)
        sp, spp = self._suppress(suppress_tokens)
        r, bufs = self._result_buffers(sl.size, max_tokens)
        temps = np.zeros(sl.size, np.float32)
        check(lib().w4j_decode_with_fallback(self._ctx, _ptr(sl), sl.size, _ptr(pr), pr.shape[1], eot, max_tokens,
                                             spp, sp.size, no_speech_token, timestamp_begin, beam_size, seed,
                                             ctypes.byref(r), _ptr(temps)))
        return self._collect(bufs, temps)

    # reference-shaped single-stream entry points
    def decode(self, encoder_output, prompt, eot_token, max_tokens, suppress_tokens=(), no_speech_token=-1,
               temperature=0.0, timestamp_begin=-1, seed=0) -> DecodeResult:
        slot = self._slot_for(encoder_output, 0)
        return self.decode_batch([slot], [list(prompt)], eot_token, max_tokens, suppress_tokens, no_speech_token,
                                 temperature, timestamp_begin, seed)[0]

    def decode_beam(self, encoder_output, prompt, eot_token, max_tokens, suppress_tokens=(), no_speech_token=-1,
                    timestamp_begin=-1, beam_size=5) -> DecodeResult:
        slot = self._slot_for(encoder_output, 0)
        return self.decode_beam_batch([slot], [list(prompt)], eot_token, max_tokens, suppress_tokens,
                                      no_speech_token, timestamp_begin, beam_size)[0]

    def decode_with_fallback(self, encoder_output, prompt, eot_token, max_tokens, suppress_tokens=(),
                             no_speech_token=-1, timestamp_begin=-1, beam_size=1, seed=0) -> DecodeResult:
        slot = self._slot_for(encoder_output, 0)
        return self.decode_with_fallback_batch([slot], [list(prompt)], eot_token, max_tokens, suppress_tokens,
                                               no_speech_token, timestamp_begin, beam_size, seed)[0]

    def cancel(self):
        check(lib().w4j_cancel(self._ctx))

    def kernel_timing(self, kernel_class: int):
        """In-chain device time of one kernel class over the next decode call: set the class (1 projections,
        2 self-attention, 3 cross-attention, 4 logits, 5 selection; 0 off), decode, then read
        ``kernel_times()``."""
        check(lib().w4j_set_kernel_timing(self._ctx, int(kernel_class)))

    def kernel_times(self):
        ms = ctypes.c_double()
        n = ctypes.c_longlong()
        check(lib().w4j_kernel_timing(self._ctx, ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    def last_timing(self):
        ms = ctypes.c_double()
        steps = ctypes.c_int()
        launches = ctypes.c_longlong()
        check(lib().w4j_last_timing(self._ctx, ctypes.byref(ms), ctypes.byref(steps), ctypes.byref(launches)))
        return ms.value, steps.value, launches.value
