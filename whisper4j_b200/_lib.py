"""ctypes binding of libwhisper4j_cuda.so (declarations in include/whisper4j_cuda.h).

The library is the only compute path: if it is missing or cannot be loaded, every
call fails loudly (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwhisper4j_cuda.so")

W4J_OK = 0
W4J_ERR_ARG = -1
W4J_ERR_STATE = -2
W4J_ERR_CUDA = -3
W4J_ERR_OOM = -4
W4J_ERR_CANCELLED = -5

GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8


class W4jError(RuntimeError):
    """Base class of library errors."""


class IllegalStateError(W4jError):
    """IllegalStateException in the reference (missing weights, no encoder output, ...)."""


class CudaError(W4jError):
    pass


class CancelledError(W4jError):
    pass


class Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "n_mels", "n_audio_ctx", "n_audio_state", "n_audio_head", "n_audio_layer",
        "n_vocab", "n_text_ctx", "n_text_state", "n_text_head", "n_text_layer")]


class TranscribeOpts(ctypes.Structure):
    _fields_ = [("sot", ctypes.POINTER(ctypes.c_int32)), ("n_sot", ctypes.c_int32), ("eot", ctypes.c_int32),
                ("no_speech", ctypes.c_int32), ("no_timestamps", ctypes.c_int32), ("sot_prev", ctypes.c_int32),
                ("ts_begin", ctypes.c_int32), ("suppress", ctypes.POINTER(ctypes.c_int32)), ("n_suppress", ctypes.c_int32),
                ("beam_size", ctypes.c_int32), ("condition_on_previous", ctypes.c_int32), ("seed", ctypes.c_uint64)]


class Segment(ctypes.Structure):
    _fields_ = [("start", ctypes.c_float), ("end", ctypes.c_float), ("token_begin", ctypes.c_int32),
                ("n_tokens", ctypes.c_int32)]


class Transcript(ctypes.Structure):
    _fields_ = [("tokens", ctypes.POINTER(ctypes.c_int32)), ("tokens_cap", ctypes.c_int32),
                ("segments", ctypes.POINTER(Segment)), ("segments_cap", ctypes.c_int32),
                ("n_tokens", ctypes.c_int32), ("n_segments", ctypes.c_int32), ("n_windows", ctypes.c_int32)]


class Result(ctypes.Structure):
    _fields_ = [("tokens", ctypes.POINTER(ctypes.c_int32)), ("lens", ctypes.POINTER(ctypes.c_int32)),
                ("sum_logprob", ctypes.POINTER(ctypes.c_double)), ("avg_logprob", ctypes.POINTER(ctypes.c_float)),
                ("compression", ctypes.POINTER(ctypes.c_float)), ("no_speech_prob", ctypes.POINTER(ctypes.c_float))]


# every symbol declared in include/whisper4j_cuda.h: name -> (restype, argtypes)
_P, _I, _F, _D, _U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_uint64
SIGNATURES = {
    "w4j_last_error": (ctypes.c_char_p, []),
    "w4j_version": (ctypes.c_char_p, []),
    "w4j_ctx_create": (_I, [ctypes.POINTER(Dims), _I, _I, _I, ctypes.POINTER(_P)]),
    "w4j_ctx_destroy": (_I, [_P]),
    "w4j_upload_tensor": (_I, [_P, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_int64), _I, _P, ctypes.c_size_t]),
    "w4j_finalize": (_I, [_P]),
    "w4j_set_encoder_output": (_I, [_P, _I, _P, _I]),
    "w4j_set_encoder_output_device": (_I, [_P, _I, _P, _I]),
    "w4j_encoder_forward": (_I, [_P, _P, _I, _P, _I]),
    "w4j_upload_mel_filters": (_I, [_P, _P, _I, _I]),
    "w4j_log_mel": (_I, [_P, _P, _I, _P]),
    "w4j_encode_audio": (_I, [_P, _P, _I, _P, _I]),
    "w4j_transcribe": (_I, [_P, _P, _I, _P, _P]),
    "w4j_forward": (_I, [_P, _I, _P, _I, _I, _P]),
    "w4j_reset_cache": (_I, [_P, _I]),
    "w4j_decode": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _I, _I, _F, _I, _U64, ctypes.POINTER(Result)]),
    "w4j_decode_beam": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _I, _I, _I, _I, ctypes.POINTER(Result)]),
    "w4j_decode_with_fallback": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _I, _I, _I, _I, _U64, ctypes.POINTER(Result),
                                      _P]),
    "w4j_cancel": (_I, [_P]),
    "w4j_compression_ratio": (_F, [_P, _I]),
    "w4j_needs_fallback": (_I, [_F, _F, _F]),
    "w4j_last_timing": (_I, [_P, ctypes.POINTER(_D), ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_longlong)]),
    "w4j_set_kernel_timing": (_I, [_P, _I]),
    "w4j_kernel_timing": (_I, [_P, ctypes.POINTER(_D), ctypes.POINTER(ctypes.c_longlong)]),
    "w4j_op_linear": (_I, [_P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _I, _P, _P]),
    "w4j_q8_0_repack": (_I, [_P, _I, _I, _P, _P]),
    "w4j_op_logits_argmax": (_I, [_P, _P, _I, _P, _I, _P, _P, _P, _P, _P]),
    "w4j_op_logits_argmax_noalloc": (_I, [_I, _P, _I, _I, _P, _I, _P, _P, _P, _P, _P]),
    "w4j_test_withhold_logits_copies": (_I, [_I]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load (once) and return the library; raises if it is absent."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise W4jError(f"{LIB_PATH} is missing: build it with `python -m whisper4j_b200.build`")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int) -> int:
    if rc >= 0:
        return rc
    msg = lib().w4j_last_error().decode(errors="replace")
    if rc == W4J_ERR_ARG:
        raise ValueError(msg)
    if rc == W4J_ERR_STATE:
        raise IllegalStateError(msg)
    if rc == W4J_ERR_OOM:
        raise MemoryError(msg)
    if rc == W4J_ERR_CANCELLED:
        raise CancelledError(msg)
    if rc == W4J_ERR_CUDA:
        raise CudaError(msg)
    raise W4jError(f"error {rc}: {msg}")
