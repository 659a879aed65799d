"""ctypes front end of the CPU oracle (oracle/w4j_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker; the product library and
its Python wrapper never import this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libw4j_oracle.so")
_lib = None
_lock = threading.Lock()


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (strict IEEE f32 flags)."""
    src = os.path.join(_HERE, "w4j_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("n_vocab", "n_audio_ctx", "n_text_ctx", "n_text_state", "n_text_head", "n_text_layer")]


class _EncDims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("n_mels", "n_audio_ctx", "n_audio_state", "n_audio_head", "n_audio_layer")]


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            P, I, F, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
            L.orc_last_error.restype = ctypes.c_char_p
            L.orc_last_loop_seconds.restype = ctypes.c_double
            L.orc_model_new.restype = P
            L.orc_model_new.argtypes = [ctypes.POINTER(_Dims)]
            L.orc_model_free.argtypes = [P]
            L.orc_set_tensor.argtypes = [P, ctypes.c_char_p, P, ctypes.c_long]
            L.orc_model_check.argtypes = [P]
            L.orc_gelu_table.restype = ctypes.POINTER(ctypes.c_float)
            L.orc_gelu_table.argtypes = [P]
            L.orc_cache_new.restype = P
            L.orc_cache_new.argtypes = [P, I]
            L.orc_cache_free.argtypes = [P]
            L.orc_cache_len.argtypes = [P]
            L.orc_forward.argtypes = [P, P, I, P, I, P, P]
            L.orc_decode.argtypes = [P, P, I, P, I, I, I, P, I, I, F, I, ctypes.c_uint64, P, P, P, P, P, I]
            L.orc_decode_beam.argtypes = [P, P, I, P, I, I, I, P, I, I, I, I, P, P, P, P, P, I]
            L.orc_set_threads.argtypes = [I]
            L.orc_set_beam_trace.argtypes = [P, ctypes.c_long]
            L.orc_beam_trace_count.restype = ctypes.c_long
            L.orc_apply_repetition_penalty.argtypes = [P, P, I, I]
            L.orc_apply_timestamp_rules.argtypes = [P, P, I, I, I, I, I]
            L.orc_dot.restype = F
            L.orc_dot.argtypes = [P, P, I]
            L.orc_matmul.argtypes = [P, P, I, I, I, P]
            L.orc_matmul_transb.argtypes = [P, P, I, I, I, F, P]
            L.orc_softmax_rows.argtypes = [P, I, I]
            L.orc_layer_norm.argtypes = [P, I, I, P, P, F, P]
            L.orc_gelu.argtypes = [P, P, ctypes.c_long]
            L.orc_f16_to_f32.restype = F
            L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
            L.orc_f32_to_f16.restype = ctypes.c_uint16
            L.orc_f32_to_f16.argtypes = [F]
            L.orc_encoder_new.restype = P
            L.orc_encoder_new.argtypes = [ctypes.POINTER(_EncDims)]
            L.orc_encoder_free.argtypes = [P]
            L.orc_encoder_set_tensor.argtypes = [P, ctypes.c_char_p, P, ctypes.c_long]
            L.orc_encoder_check.argtypes = [P]
            L.orc_encoder_forward.argtypes = [P, P, P]
            L.orc_log_mel.argtypes = [P, I, P, I, I, I, I, P]
            _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


class OracleError(RuntimeError):
    pass


def _check(rc):
    if rc < 0:
        raise OracleError(lib().orc_last_error().decode())


def set_threads(n: int) -> None:
    """Threads of the oracle's own loops (1 = the reference's single-threaded decoder)."""
    lib().orc_set_threads(int(n))


# ---- tensor KATs ------------------------------------------------------------

def dot(a, b) -> float:
    a, b = _f32(a), _f32(b)
    return float(lib().orc_dot(_p(a), _p(b), a.size))


def matmul(a, b):
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    N = b.shape[1]
    out = np.zeros((M, N), np.float32)
    lib().orc_matmul(_p(a), _p(b), M, K, N, _p(out))
    return out


def matmul_transb(a, b, alpha=1.0):
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    N = b.shape[0]
    out = np.zeros((M, N), np.float32)
    lib().orc_matmul_transb(_p(a), _p(b), M, K, N, alpha, _p(out))
    return out


def softmax(x):
    x = _f32(x).copy()
    rows = x.size // x.shape[-1]
    lib().orc_softmax_rows(_p(x), rows, x.shape[-1])
    return x


def layer_norm(x, g, b, eps=1e-5):
    x, g, b = _f32(x), _f32(g), _f32(b)
    y = np.zeros_like(x)
    lib().orc_layer_norm(_p(x), x.size // x.shape[-1], x.shape[-1], _p(g), _p(b), eps, _p(y))
    return y


def f32_to_f16_bits(v: float) -> int:
    return int(lib().orc_f32_to_f16(v))


# ---- model ------------------------------------------------------------------

class OracleModel:
    """The oracle's decoder, loaded from a parsed GGML model (whisper4j_b200.ggml.GgmlModel)."""

    def __init__(self, gmodel, n_audio_ctx: int | None = None):
        from whisper4j_b200 import ggml  # dequantisation helper with the reference's semantics

        dm = gmodel.dims
        self.dims = dm
        self.n_audio_ctx = n_audio_ctx or dm.n_audio_ctx
        d = _Dims(dm.n_vocab, self.n_audio_ctx, dm.n_text_ctx, dm.n_text_state, dm.n_text_head, dm.n_text_layer)
        self._m = lib().orc_model_new(ctypes.byref(d))
        if not self._m:
            raise OracleError(lib().orc_last_error().decode())
        for name, t in gmodel.tensors.items():
            if not name.startswith("decoder."):
                continue
            arr = _f32(ggml.dequantize(t)).reshape(-1)
            _check(lib().orc_set_tensor(self._m, name.encode(), _p(arr), arr.size))
        _check(lib().orc_model_check(self._m))

    def close(self):
        if self._m:
            lib().orc_model_free(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def gelu_table(self) -> np.ndarray:
        ptr = lib().orc_gelu_table(self._m)
        return np.ctypeslib.as_array(ptr, shape=(65536,)).copy()

    def gelu(self, x):
        x = _f32(x).copy()
        lib().orc_gelu(self._m, _p(x), x.size)
        return x

    def new_cache(self):
        return OracleCache(self)

    def forward(self, tokens, xa, cache=None) -> np.ndarray:
        """WhisperDecoder.forward: logits (n, n_vocab) as float32."""
        tok = _i32(tokens)
        xa = _f32(xa)
        V = self.dims.n_vocab
        out = np.zeros((tok.size, V), np.float32)
        _check(lib().orc_forward(self._m, _p(tok), tok.size, _p(xa), xa.shape[0],
                                 cache._c if cache is not None else None, _p(out)))
        return out

    def decode(self, xa, prompt, eot, max_tokens, suppress=(), no_speech=-1, temperature=0.0, ts_begin=-1,
               seed=0, max_steps=0):
        xa, pr, sp = _f32(xa), _i32(prompt), _i32(list(suppress) or [0])
        toks = np.zeros(max(max_tokens, 1), np.int32)
        n = ctypes.c_int()
        s = ctypes.c_double()
        a = ctypes.c_float()
        ns = ctypes.c_float()
        _check(lib().orc_decode(self._m, _p(xa), xa.shape[0], _p(pr), pr.size, eot, max_tokens, _p(sp),
                                len(suppress), no_speech, temperature, ts_begin, seed, _p(toks), ctypes.byref(n),
                                ctypes.byref(s), ctypes.byref(a), ctypes.byref(ns), max_steps))
        return dict(tokens=toks[:n.value].tolist(), sum_logprob=s.value, avg_logprob=a.value,
                    no_speech_prob=ns.value, loop_seconds=lib().orc_last_loop_seconds())

    def decode_beam(self, xa, prompt, eot, max_tokens, suppress=(), no_speech=-1, ts_begin=-1, beam=5,
                    max_steps=0, trace=False):
        """WhisperDecoder.decodeBeam.  trace=True adds ``trace``: every ranked candidate of every step
        as rows (step, parent beam, token, score, outcome) — outcome is the new beam index when
        kept, -2 when the candidate finished a sequence, -1 when dropped or not reached."""
        xa, pr, sp = _f32(xa), _i32(prompt), _i32(list(suppress) or [0])
        toks = np.zeros(max(max_tokens, 1) + 1, np.int32)
        n = ctypes.c_int()
        s = ctypes.c_double()
        a = ctypes.c_float()
        ns = ctypes.c_float()
        tbuf = np.zeros(((max_tokens + 1) * beam * (beam + 1) + beam, 5), np.float64) if trace else None
        if trace:
            lib().orc_set_beam_trace(_p(tbuf), tbuf.shape[0])
        try:
            _check(lib().orc_decode_beam(self._m, _p(xa), xa.shape[0], _p(pr), pr.size, eot, max_tokens, _p(sp),
                                         len(suppress), no_speech, ts_begin, beam, _p(toks), ctypes.byref(n),
                                         ctypes.byref(s), ctypes.byref(a), ctypes.byref(ns), max_steps))
        finally:
            count = lib().orc_beam_trace_count() if trace else 0
            if trace:
                lib().orc_set_beam_trace(None, 0)
        out = dict(tokens=toks[:n.value].tolist(), sum_logprob=s.value, avg_logprob=a.value,
                   no_speech_prob=ns.value, loop_seconds=lib().orc_last_loop_seconds())
        if trace:
            out["trace"] = tbuf[:count].copy()
        return out


class OracleCache:
    def __init__(self, model: OracleModel):
        self._model = model
        self._c = lib().orc_cache_new(model._m, model.n_audio_ctx)

    def __len__(self):
        return lib().orc_cache_len(self._c)

    def __del__(self):
        try:
            lib().orc_cache_free(self._c)
        except Exception:
            pass


def apply_repetition_penalty(logits, generated):
    lg = _f32(logits).copy()
    g = _i32(list(generated) or [0])
    lib().orc_apply_repetition_penalty(_p(lg), _p(g), len(generated), lg.size)
    return lg


def apply_timestamp_rules(logits, generated, ts_begin, eot, is_first):
    lg = _f32(logits).copy()
    g = _i32(list(generated) or [0])
    lib().orc_apply_timestamp_rules(_p(lg), _p(g), len(generated), ts_begin, eot, lg.size, int(is_first))
    return lg


class OracleEncoder:
    """The oracle's audio encoder (WhisperEncoder.forward), loaded from a parsed GGML model with
    encoder tensors."""

    def __init__(self, gmodel):
        from whisper4j_b200 import ggml

        dm = gmodel.dims
        self.dims = dm
        d = _EncDims(dm.n_mels, dm.n_audio_ctx, dm.n_audio_state, dm.n_audio_head, dm.n_audio_layer)
        self._e = lib().orc_encoder_new(ctypes.byref(d))
        if not self._e:
            raise OracleError(lib().orc_last_error().decode())
        for name, t in gmodel.tensors.items():
            if name.startswith("encoder."):
                arr = _f32(ggml.dequantize(t)).reshape(-1)
                _check(lib().orc_encoder_set_tensor(self._e, name.encode(), _p(arr), arr.size))
        _check(lib().orc_encoder_check(self._e))

    def forward(self, mel) -> np.ndarray:
        """mel: (n_mels, 2 n_audio_ctx) -> encoder output xa (n_audio_ctx, n_audio_state)."""
        dm = self.dims
        m = _f32(mel)
        if m.shape != (dm.n_mels, 2 * dm.n_audio_ctx):
            raise ValueError(f"mel must be ({dm.n_mels}, {2 * dm.n_audio_ctx}), got {m.shape}")
        out = np.empty((dm.n_audio_ctx, dm.n_audio_state), np.float32)
        _check(lib().orc_encoder_forward(self._e, _p(m), _p(out)))
        return out

    def close(self):
        if self._e:
            lib().orc_encoder_free(self._e)
            self._e = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def log_mel(audio, filters, out_frames: int, hop: int = 160) -> np.ndarray:
    """FeatureExtractor.extract + padOrTrim: (n_mels, out_frames) log-mel of 16 kHz samples with the
    model's filters (n_mels, n_bins)."""
    a = _f32(audio).reshape(-1)
    f = _f32(filters)
    n_mels, n_bins = f.shape
    out = np.empty((n_mels, out_frames), np.float32)
    _check(lib().orc_log_mel(_p(a) if a.size else None, a.size, _p(f), n_mels, n_bins, hop, out_frames, _p(out)))
    return out


# ---------------------------------------------------------------------------
# the chunked transcription loop (WhisperModel.transcribeChunked, WhisperModel.java:334-427)
# ---------------------------------------------------------------------------
def f32(x) -> float:
    return float(np.float32(x))


def timestamp_segments(tokens, ts_begin, offset, precision):
    """parseTimestampSegments (WhisperModel.java:430-490): [(start, end, text_tokens)], segments with
    at least one text token."""
    offset, precision = np.float32(offset), np.float32(precision)
    ts = [i for i, t in enumerate(tokens) if t >= ts_begin]
    out = []
    if len(ts) < 2:
        text = [t for t in tokens if t < ts_begin]
        if text:
            end = offset + np.float32(30.0) if not ts else offset + np.float32(tokens[ts[0]] - ts_begin) * precision
            out.append((f32(offset), f32(end), text))
        return out
    last = 0
    for i in range(len(ts) - 1):
        if ts[i + 1] != ts[i] + 1:
            continue
        sl = tokens[last:ts[i + 1]]
        start, end = offset, offset + np.float32(30.0)
        for t in sl:
            if t >= ts_begin:
                start = offset + np.float32(t - ts_begin) * precision
                break
        for t in reversed(sl):
            if t >= ts_begin:
                end = offset + np.float32(t - ts_begin) * precision
                break
        text = [t for t in sl if t < ts_begin]
        if text:
            out.append((f32(start), f32(end), text))
        last = ts[i + 1]
    return out


def prompt_with_context(base, prev, sot_prev, n_text_ctx, condition):
    """buildPromptWithContext (WhisperModel.java:507-530)."""
    if not condition or not prev:
        return list(base)
    max_prev = (n_text_ctx // 2 - 1) - len(base) - 1
    if max_prev <= 0:
        return list(base)
    n = min(len(prev), max_prev)
    return [sot_prev] + list(prev[len(prev) - n:]) + list(base)


def transcribe_chunked(n_samples, n_audio_ctx, n_text_ctx, sot, no_timestamps, sot_prev, ts_begin,
                       condition_on_previous, window, decode):
    """The loop of WhisperModel.transcribeChunked over injected stages: window(a0, n_valid) prepares
    the 30 s window at sample a0 (front end + encoder), decode(prompt, max_tokens) -> (tokens,
    avg_logprob, no_speech_prob) runs decodeWithFallback on it.  Returns [(start, end, tokens)]."""
    n_frames = 2 * n_audio_ctx
    stride, hop = n_frames // n_audio_ctx, 160
    chunk = n_frames * hop
    precision = np.float32(stride) * np.float32(160.0) / np.float32(16000.0)
    total = int(np.float32(n_samples) / np.float32(160.0))
    duration = np.float32(n_samples) / np.float32(16000.0)
    with_ts = ts_begin > 0
    base = list(sot) + ([] if with_ts else [no_timestamps])
    prev, segs, seek = [], [], 0
    while seek < total:
        offset = np.float32(seek) * np.float32(160.0) / np.float32(16000.0)
        seg_size = min(n_frames, total - seek)
        a0 = seek * hop
        window(a0, max(min(n_samples - a0, chunk), 0))
        max_tokens = n_text_ctx // 2
        if seg_size < n_frames:
            max_tokens = max(8, max_tokens * seg_size // n_frames)
        tokens, avg, nsp = decode(prompt_with_context(base, prev, sot_prev, n_text_ctx, condition_on_previous),
                                  max_tokens)
        if condition_on_previous and prev and avg < -1.0:
            tokens, avg, nsp = decode(base, max_tokens)
            prev = []
        if nsp > 0.6 and avg < -1.0:
            seek += seg_size
            continue
        if with_ts:
            segs += timestamp_segments(tokens, ts_begin, offset, precision)
            last = next((t - ts_begin for t in reversed(tokens) if t >= ts_begin), -1)
            seek += max(last * stride, stride) if last > 0 else seg_size
        else:
            if tokens:
                segs.append((f32(offset), f32(min(offset + np.float32(seg_size) * np.float32(160.0) / np.float32(16000.0),
                                                   duration)), list(tokens)))
            seek += seg_size
        if condition_on_previous:
            prev = list(tokens)
    return segs
