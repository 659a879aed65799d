"""GGML file format: writer/parser round trip and the reference loader's semantics (GgmlLoader.java)."""
import struct

import numpy as np
import pytest

from whisper4j_b200 import ggml

from .helpers import SMALL, model_bytes


def test_round_trip_header_and_tensors():
    buf = model_bytes(SMALL, 5)
    m = ggml.parse(buf)
    assert m.dims == SMALL
    assert m.mel_filters.shape == (SMALL.n_mels, 201)
    names = [n for n, _, _ in ggml.decoder_tensor_specs(SMALL)]
    assert list(m.tensors) == names
    te = m.tensors["decoder.token_embedding.weight"]
    assert te.ne == (SMALL.n_text_state, SMALL.n_vocab) and te.shape == (SMALL.n_vocab, SMALL.n_text_state)
    assert te.ttype == ggml.GGML_TYPE_F16
    assert m.tensors["decoder.positional_embedding"].ttype == ggml.GGML_TYPE_F32
    assert "decoder.blocks.0.attn.key.bias" not in m.tensors  # key bias is absent (WhisperEncoder.java:101)


def test_dequantize_f16_exact():
    m = ggml.parse(model_bytes(SMALL, 5))
    t = m.tensors["decoder.blocks.1.mlp.0.weight"]
    v = ggml.dequantize(t)
    assert v.shape == (4 * SMALL.n_text_state, SMALL.n_text_state)
    raw = np.frombuffer(t.data, dtype="<f2").reshape(v.shape)
    np.testing.assert_array_equal(v, raw.astype(np.float32))


def test_q8_0_known_answer():
    # one block: scale f16(0.5), quants -128..127 pattern -> value = q * scale (GgmlLoader.java:292-300)
    q = np.array([-128, -1, 0, 1, 127] + list(range(-13, 14)), np.int8)[:32]
    blk = np.float16(0.5).tobytes() + q.tobytes()
    t = ggml.GgmlTensor("x", ggml.GGML_TYPE_Q8_0, (32,), memoryview(blk))
    np.testing.assert_array_equal(ggml.dequantize(t), q.astype(np.float32) * np.float32(0.5))


def test_q8_0_quantize_round_trip():
    rng = np.random.default_rng(1)
    w = rng.standard_normal((4, 64)).astype(np.float32) * 0.02
    blocks = ggml.quantize_q8_0(w)
    assert len(blocks) == 8 * 34
    t = ggml.GgmlTensor("w", ggml.GGML_TYPE_Q8_0, (64, 4), memoryview(blocks))
    back = ggml.dequantize(t)
    amax = np.abs(w.reshape(-1, 32)).max(axis=1).repeat(32).reshape(w.shape)
    assert np.all(np.abs(back - w) <= amax / 127 * 0.5 + 1e-6)


@pytest.mark.parametrize("ttype,n,size", [(0, 64, 256), (1, 64, 128), (2, 64, 36), (3, 64, 40), (6, 64, 44),
                                          (7, 64, 48), (8, 64, 68)])
def test_tensor_data_size(ttype, n, size):  # GgmlLoader.java:302-313
    assert ggml.tensor_data_size(ttype, n) == size


def test_bad_magic():
    with pytest.raises(ValueError, match="not a GGML file"):
        ggml.parse(b"\0" * 64)


def test_truncated_tensor_data():
    buf = model_bytes(SMALL, 5)
    with pytest.raises(ValueError, match="truncated"):
        ggml.parse(buf[:-10])


def test_invalid_tensor_header_ends_list():
    # GgmlLoader.java:153-158: an implausible header ends the tensor list without an error
    buf = bytearray(model_bytes(SMALL, 5)) + struct.pack("<3i", 9, 1, 0)
    m = ggml.parse(bytes(buf))
    assert len(m.tensors) == len(list(ggml.decoder_tensor_specs(SMALL)))


def test_q8_model_types():
    m = ggml.parse(model_bytes(SMALL, 6, "q8_0"))
    assert m.tensors["decoder.blocks.0.attn.query.weight"].ttype == ggml.GGML_TYPE_Q8_0
    assert m.tensors["decoder.token_embedding.weight"].ttype == ggml.GGML_TYPE_F16
    assert m.tensors["decoder.blocks.0.mlp_ln.weight"].ttype == ggml.GGML_TYPE_F16
