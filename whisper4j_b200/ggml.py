"""Whisper GGML (legacy whisper.cpp) model files: parse, write, and seeded synthetic models.

The parser follows the reference loader byte for byte (model/GgmlLoader.java:95-220):
magic 0x67676d6c, eleven int32 hyper-parameters (:101-112), the mel filter bank
(:120-124), the vocabulary (:127-139) and then tensors with the header
``{n_dims, name_len, ttype, ne[n_dims], name}`` and no alignment padding
(:148-203).  ``ne`` is fastest-dimension first, so the row-major shape is ``ne``
reversed (:180-183).  Tensor payload sizes follow ``tensorDataSize`` (:302-313).

Unlike the reference, which dequantises every tensor to f32 on the heap
(:185-202, :224-300), the parser hands out the raw payload bytes; the device
library takes f16 and Q8_0 as stored (``w4j_upload_tensor``).
"""
from __future__ import annotations

import dataclasses
import struct
from typing import Iterable

import numpy as np

GGML_MAGIC = 0x67676D6C
GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_0 = 2
GGML_TYPE_Q4_1 = 3
GGML_TYPE_Q5_0 = 6
GGML_TYPE_Q5_1 = 7
GGML_TYPE_Q8_0 = 8

_BLOCK_BYTES = {GGML_TYPE_Q4_0: 18, GGML_TYPE_Q4_1: 20, GGML_TYPE_Q5_0: 22, GGML_TYPE_Q5_1: 24, GGML_TYPE_Q8_0: 34}


@dataclasses.dataclass(frozen=True)
class ModelDimensions:
    """model/ModelDimensions.java:6-17 (same field order as the GGML header is read)."""

    n_mels: int
    n_audio_ctx: int
    n_audio_state: int
    n_audio_head: int
    n_audio_layer: int
    n_vocab: int
    n_text_ctx: int
    n_text_state: int
    n_text_head: int
    n_text_layer: int


# Architectures named by the benchmark configurations (ModelDimensions of the public checkpoints).
ARCHS = {
    "tiny.en": ModelDimensions(80, 1500, 384, 6, 4, 51864, 448, 384, 6, 4),
    "base.en": ModelDimensions(80, 1500, 512, 8, 6, 51864, 448, 512, 8, 6),
    "small": ModelDimensions(80, 1500, 768, 12, 12, 51865, 448, 768, 12, 12),
    "large-v3-turbo": ModelDimensions(128, 1500, 1280, 20, 32, 51866, 448, 1280, 20, 4),
    "large-v3": ModelDimensions(128, 1500, 1280, 20, 32, 51866, 448, 1280, 20, 32),
}


def tensor_data_size(ttype: int, n_elements: int) -> int:
    """GgmlLoader.java:302-313."""
    if ttype == GGML_TYPE_F32:
        return n_elements * 4
    if ttype == GGML_TYPE_F16:
        return n_elements * 2
    if ttype in _BLOCK_BYTES:
        return (n_elements // 32) * _BLOCK_BYTES[ttype]
    raise ValueError(f"unsupported GGML type: {ttype}")


@dataclasses.dataclass
class GgmlTensor:
    name: str
    ttype: int
    ne: tuple  # fastest dimension first, as stored
    data: memoryview  # raw payload bytes

    @property
    def shape(self) -> tuple:
        return tuple(reversed(self.ne))

    @property
    def n_elements(self) -> int:
        n = 1
        for v in self.ne:
            n *= v
        return n


@dataclasses.dataclass
class GgmlModel:
    dims: ModelDimensions
    ftype: int
    mel_filters: np.ndarray
    vocab: list
    tensors: dict  # name -> GgmlTensor, in file order


def parse(buf) -> GgmlModel:
    """Parse a whole GGML file held in ``buf`` (bytes, bytearray, mmap or memoryview)."""
    mv = memoryview(buf).cast("B")
    size = len(mv)
    pos = 0

    def i32():
        nonlocal pos
        if pos + 4 > size:
            raise ValueError("truncated GGML header")
        v = struct.unpack_from("<i", mv, pos)[0]
        pos += 4
        return v

    magic = i32() & 0xFFFFFFFF
    if magic != GGML_MAGIC:
        raise ValueError("not a GGML file (magic: 0x%08X)" % magic)
    hp = [i32() for _ in range(11)]
    n_vocab, n_audio_ctx, n_audio_state, n_audio_head, n_audio_layer = hp[:5]
    n_text_ctx, n_text_state, n_text_head, n_text_layer, n_mels, ftype = hp[5:]
    dims = ModelDimensions(n_mels, n_audio_ctx, n_audio_state, n_audio_head, n_audio_layer,
                           n_vocab, n_text_ctx, n_text_state, n_text_head, n_text_layer)
    n_mel = i32()
    n_fft = i32()
    if n_mel < 0 or n_fft < 0 or pos + n_mel * n_fft * 4 > size:
        raise ValueError("truncated GGML mel filters")
    mel = np.frombuffer(mv, dtype="<f4", count=n_mel * n_fft, offset=pos).reshape(n_mel, n_fft).copy()
    pos += n_mel * n_fft * 4
    vocab_count = i32()
    vocab = []
    for _ in range(vocab_count):
        ln = i32()
        if ln > 0:
            if pos + ln > size:
                raise ValueError("truncated GGML vocabulary")
            vocab.append(bytes(mv[pos:pos + ln]).decode("utf-8", errors="replace"))
            pos += ln
        else:
            vocab.append("")
    tensors = {}
    while pos + 12 <= size:
        n_dims, name_len, ttype = struct.unpack_from("<3i", mv, pos)
        # GgmlLoader.java:153-158: an implausible header ends the tensor list
        if n_dims < 1 or n_dims > 4 or name_len < 1 or name_len > 256 or ttype < 0 or ttype > 15:
            break
        pos += 12
        if pos + 4 * n_dims + name_len > size:
            raise ValueError("truncated GGML tensor header")
        ne = struct.unpack_from("<%di" % n_dims, mv, pos)
        pos += 4 * n_dims
        name = bytes(mv[pos:pos + name_len]).decode("utf-8").strip()
        pos += name_len
        n_el = 1
        for v in ne:
            n_el *= v
        nbytes = tensor_data_size(ttype, n_el)
        if pos + nbytes > size:
            raise ValueError(f"truncated GGML tensor data: {name}")
        tensors[name] = GgmlTensor(name, ttype, tuple(ne), mv[pos:pos + nbytes])
        pos += nbytes
    return GgmlModel(dims, ftype, mel, vocab, tensors)


def load(path) -> GgmlModel:
    """Read a GGML file into memory and parse it (GgmlLoader.load, :50-70)."""
    with open(path, "rb") as f:
        data = f.read()
    return parse(data)


# ----------------------------------------------------------------------------
# dequantisation (reference semantics, used by the CPU oracle and by tests)
# ----------------------------------------------------------------------------

def dequantize(t: GgmlTensor) -> np.ndarray:
    """f32 values in row-major ``t.shape`` (GgmlLoader.java:224-238, Q8_0 :292-300)."""
    n = t.n_elements
    if t.ttype == GGML_TYPE_F32:
        out = np.frombuffer(t.data, dtype="<f4", count=n).astype(np.float32)
    elif t.ttype == GGML_TYPE_F16:
        out = np.frombuffer(t.data, dtype="<f2", count=n).astype(np.float32)
    elif t.ttype == GGML_TYPE_Q8_0:
        blocks = np.frombuffer(t.data, dtype=np.uint8, count=(n // 32) * 34).reshape(-1, 34)
        scale = blocks[:, :2].copy().view("<f2").astype(np.float32)  # (nb, 1)
        q = blocks[:, 2:].view(np.int8).astype(np.float32)
        out = (q * scale).reshape(-1)  # byte promoted to float, times float scale
    else:
        raise ValueError(f"unsupported GGML type for this path: {t.ttype}")
    return out.reshape(t.shape)


def quantize_q8_0(w: np.ndarray) -> bytes:
    """Q8_0 blocks of 32: f16 scale max|w|/127 then 32 int8 round-half-away-from-zero(w/scale)."""
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(flat).max(axis=1)
    d = amax / 127.0
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1.0), 0.0).astype(np.float32)
    v = flat * inv[:, None]
    q = (np.sign(v) * np.floor(np.abs(v) + 0.5)).clip(-127, 127).astype(np.int8)
    out = np.empty((flat.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.astype("<f2").reshape(-1, 1).view(np.uint8)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


# ----------------------------------------------------------------------------
# writer and seeded synthetic models
# ----------------------------------------------------------------------------

def _encode_tensor(name: str, arr: np.ndarray, ttype: int) -> bytes:
    shape = arr.shape
    ne = tuple(reversed(shape))
    nb = name.encode("utf-8")
    head = struct.pack("<3i", len(ne), len(nb), ttype) + struct.pack("<%di" % len(ne), *ne) + nb
    if ttype == GGML_TYPE_F32:
        body = np.ascontiguousarray(arr, dtype="<f4").tobytes()
    elif ttype == GGML_TYPE_F16:
        body = np.ascontiguousarray(arr, dtype="<f2").tobytes()
    elif ttype == GGML_TYPE_Q8_0:
        if arr.size % 32:
            raise ValueError(f"{name}: Q8_0 needs a multiple of 32 elements")
        body = quantize_q8_0(arr)
    else:
        raise ValueError(f"writer does not produce ttype {ttype}")
    return head + body


def write(dims: ModelDimensions, tensors: Iterable, ftype: int = 1, mel_filters: np.ndarray | None = None,
          vocab: list | None = None) -> bytes:
    """Serialise ``tensors`` = iterable of (name, f32/f16 array, ttype) as a GGML file."""
    parts = [struct.pack("<I", GGML_MAGIC),
             struct.pack("<11i", dims.n_vocab, dims.n_audio_ctx, dims.n_audio_state, dims.n_audio_head,
                         dims.n_audio_layer, dims.n_text_ctx, dims.n_text_state, dims.n_text_head,
                         dims.n_text_layer, dims.n_mels, ftype)]
    if mel_filters is None:
        mel_filters = np.zeros((dims.n_mels, 201), dtype=np.float32)
    parts.append(struct.pack("<2i", *mel_filters.shape))
    parts.append(np.ascontiguousarray(mel_filters, dtype="<f4").tobytes())
    vocab = vocab if vocab is not None else [bytes([i]).decode("latin-1") for i in range(256)]
    parts.append(struct.pack("<i", len(vocab)))
    for tok in vocab:
        b = tok.encode("utf-8")
        parts.append(struct.pack("<i", len(b)) + b)
    for name, arr, ttype in tensors:
        parts.append(_encode_tensor(name, arr, ttype))
    return b"".join(parts)


def mel_filterbank(n_mels: int, n_fft: int = 400, sr: int = 16000) -> np.ndarray:
    """Slaney-style triangular mel filters (n_mels, n_fft//2+1) for synthetic model files."""
    def hz_to_mel(f):
        f = np.asarray(f, dtype=np.float64)
        lin = f / (200.0 / 3)
        log = 15.0 + np.log(np.maximum(f, 1e-10) / 1000.0) / (np.log(6.4) / 27.0)
        return np.where(f >= 1000.0, log, lin)

    def mel_to_hz(m):
        m = np.asarray(m, dtype=np.float64)
        lin = m * (200.0 / 3)
        log = 1000.0 * np.exp((np.log(6.4) / 27.0) * (m - 15.0))
        return np.where(m >= 15.0, log, lin)

    n_bins = n_fft // 2 + 1
    freqs = np.linspace(0, sr / 2, n_bins)
    mpts = np.linspace(hz_to_mel(0.0), hz_to_mel(sr / 2), n_mels + 2)
    hz = mel_to_hz(mpts)
    fb = np.zeros((n_mels, n_bins))
    for i in range(n_mels):
        lo, c, hi = hz[i], hz[i + 1], hz[i + 2]
        up = (freqs - lo) / max(c - lo, 1e-9)
        down = (hi - freqs) / max(hi - c, 1e-9)
        fb[i] = np.maximum(0, np.minimum(up, down)) * (2.0 / (hi - lo))
    return fb.astype(np.float32)


def decoder_tensor_specs(dims: ModelDimensions):
    """(name, shape, kind) of every decoder tensor; kind in {'matrix','embed','pos','ln_w','ln_b','bias'}.

    Names follow WhisperDecoder.java:36-56, :658-669 and WhisperEncoder.buildMHA (key bias absent).
    """
    d, V, C = dims.n_text_state, dims.n_vocab, dims.n_text_ctx
    yield "decoder.token_embedding.weight", (V, d), "embed"
    yield "decoder.positional_embedding", (C, d), "pos"
    for i in range(dims.n_text_layer):
        p = f"decoder.blocks.{i}."
        for att in ("attn", "cross_attn"):
            yield p + f"{att}.query.weight", (d, d), "matrix"
            yield p + f"{att}.query.bias", (d,), "bias"
            yield p + f"{att}.key.weight", (d, d), "matrix"
            yield p + f"{att}.value.weight", (d, d), "matrix"
            yield p + f"{att}.value.bias", (d,), "bias"
            yield p + f"{att}.out.weight", (d, d), "matrix"
            yield p + f"{att}.out.bias", (d,), "bias"
            yield p + f"{att}_ln.weight", (d,), "ln_w"
            yield p + f"{att}_ln.bias", (d,), "ln_b"
        yield p + "mlp.0.weight", (4 * d, d), "matrix"
        yield p + "mlp.0.bias", (4 * d,), "bias"
        yield p + "mlp.2.weight", (d, 4 * d), "matrix"
        yield p + "mlp.2.bias", (d,), "bias"
        yield p + "mlp_ln.weight", (d,), "ln_w"
        yield p + "mlp_ln.bias", (d,), "ln_b"
    yield "decoder.ln.weight", (d,), "ln_w"
    yield "decoder.ln.bias", (d,), "ln_b"


def encoder_tensor_specs(dims: ModelDimensions):
    """Encoder tensors (WhisperEncoder.java:27-39, :86-105); conv biases stored as ne=[1, out]."""
    d, nm = dims.n_audio_state, dims.n_mels
    yield "encoder.conv1.weight", (d, nm, 3), "matrix"
    yield "encoder.conv1.bias", (d, 1), "bias"
    yield "encoder.conv2.weight", (d, d, 3), "matrix"
    yield "encoder.conv2.bias", (d, 1), "bias"
    yield "encoder.positional_embedding", (dims.n_audio_ctx, d), "pos"
    for i in range(dims.n_audio_layer):
        p = f"encoder.blocks.{i}."
        yield p + "attn.query.weight", (d, d), "matrix"
        yield p + "attn.query.bias", (d,), "bias"
        yield p + "attn.key.weight", (d, d), "matrix"
        yield p + "attn.value.weight", (d, d), "matrix"
        yield p + "attn.value.bias", (d,), "bias"
        yield p + "attn.out.weight", (d, d), "matrix"
        yield p + "attn.out.bias", (d,), "bias"
        yield p + "attn_ln.weight", (d,), "ln_w"
        yield p + "attn_ln.bias", (d,), "ln_b"
        yield p + "mlp.0.weight", (4 * d, d), "matrix"
        yield p + "mlp.0.bias", (4 * d,), "bias"
        yield p + "mlp.2.weight", (d, 4 * d), "matrix"
        yield p + "mlp.2.bias", (d,), "bias"
        yield p + "mlp_ln.weight", (d,), "ln_w"
        yield p + "mlp_ln.bias", (d,), "ln_b"
    yield "encoder.ln_post.weight", (d,), "ln_w"
    yield "encoder.ln_post.bias", (d,), "ln_b"


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> np.ndarray:
    """Sinusoidal position table (the encoder's fixed positional embedding)."""
    inc = np.log(max_timescale) / (channels // 2 - 1)
    inv = np.exp(-inc * np.arange(channels // 2))
    t = np.arange(length)[:, None] * inv[None, :]
    return np.concatenate([np.sin(t), np.cos(t)], axis=1).astype(np.float32)


def synthetic_tensors(dims: ModelDimensions, seed: int, wtype: str = "f16", include_encoder: bool = False,
                      std: float = 0.02, bias_std: float = 0.0, ln_std: float = 0.0):
    """Seeded random-init tensors: matrices N(0, std) stored f16 or Q8_0; LayerNorm gamma=1 beta=0;
    biases 0 (optionally N(0, bias_std) / gamma 1+N(0, ln_std) for stronger parity tests).

    Matrices are drawn in spec order from numpy's PCG64 stream seeded with ``seed``; Q8_0 models keep
    the token embedding in f16 (it is also the logits matrix) and the LayerNorm parameters in f16.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    q8 = wtype == "q8_0"
    specs = list(decoder_tensor_specs(dims))
    if include_encoder:
        specs = list(encoder_tensor_specs(dims)) + specs
    for name, shape, kind in specs:
        if kind in ("matrix", "embed"):
            arr = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
            if kind == "matrix" and q8 and not name.startswith("encoder.conv"):
                yield name, arr, GGML_TYPE_Q8_0
            else:
                yield name, arr.astype(np.float16), GGML_TYPE_F16
        elif kind == "pos":
            if name.startswith("encoder."):
                yield name, sinusoids(*shape), GGML_TYPE_F32
            else:
                arr = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
                yield name, arr, GGML_TYPE_F32
        elif kind == "ln_w":
            arr = np.ones(shape, dtype=np.float32)
            if ln_std:
                arr = arr + rng.standard_normal(shape, dtype=np.float32) * np.float32(ln_std)
            yield name, arr.astype(np.float16) if q8 else arr, GGML_TYPE_F16 if q8 else GGML_TYPE_F32
        elif kind == "ln_b":
            arr = np.zeros(shape, dtype=np.float32)
            if ln_std:
                arr = arr + rng.standard_normal(shape, dtype=np.float32) * np.float32(ln_std)
            yield name, arr.astype(np.float16) if q8 else arr, GGML_TYPE_F16 if q8 else GGML_TYPE_F32
        else:  # bias
            arr = np.zeros(shape, dtype=np.float32)
            if bias_std:
                arr = arr + rng.standard_normal(shape, dtype=np.float32) * np.float32(bias_std)
            yield name, arr, GGML_TYPE_F32


def synthetic_model_bytes(dims: ModelDimensions, seed: int, wtype: str = "f16", include_encoder: bool = False,
                          **kw) -> bytes:
    ftype = {"f16": 1, "q8_0": 7}[wtype]  # whisper.cpp ftype codes (7 = mostly Q8_0)
    return write(dims, synthetic_tensors(dims, seed, wtype, include_encoder, **kw), ftype=ftype,
                 mel_filters=mel_filterbank(dims.n_mels))
