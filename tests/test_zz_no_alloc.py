"""w4j_op_logits_argmax_noalloc: the vocabulary pass (LN -> logits -> argmax + log-softmax) without
a context and without any device allocation, its per-block partials in a static device array.

It must return what w4j_op_logits_argmax returns on the same inputs (the final LayerNorm and
tied-embedding logits of WhisperDecoder.java:102-103, argmax :566-574, logSoftmax :614-626).
The file name sorts last so that the suite also runs it after every other test used the device;
it creates everything it needs itself, so it passes alone too.
"""
import ctypes

import numpy as np
import pytest

from whisper4j_b200 import ggml
from whisper4j_b200._lib import W4J_ERR_ARG, check, lib
from whisper4j_b200.decoder import WhisperDecoder

MAX_ROWS = 16  # W4J_NOALLOC_MAX_ROWS
V = 51864


def _call(device, x, M, d, E, Vv, g, b, tok, lp):
    return lib().w4j_op_logits_argmax_noalloc(device, x, M, d, E, Vv, g, b, tok, lp, None)


def test_rejects_out_of_range_before_device_use():
    p = ctypes.c_void_p(256)  # aligned dummy; the checks run before any device call
    for M in (0, MAX_ROWS + 1):
        assert _call(0, p, M, 384, p, V, p, p, p, p) == W4J_ERR_ARG
        assert b"static" in lib().w4j_last_error() and b"16" in lib().w4j_last_error()
    assert _call(0, p, 1, 100, p, V, p, p, p, p) == W4J_ERR_ARG
    assert b"multiple of 64" in lib().w4j_last_error()
    assert _call(0, ctypes.c_void_p(260), 1, 384, p, V, p, p, p, p) == W4J_ERR_ARG
    assert b"aligned" in lib().w4j_last_error()
    assert _call(0, None, 1, 384, p, V, p, p, p, p) == W4J_ERR_ARG


@pytest.fixture(scope="module")
def vocab_ctx():
    """A one-layer d=384 model with the full Whisper vocabulary: the context of the existing op."""
    pytest.importorskip("torch")
    dims = ggml.ModelDimensions(80, 16, 384, 6, 1, V, 16, 384, 6, 1)
    d = WhisperDecoder(ggml.parse(ggml.synthetic_model_bytes(dims, 7)), max_streams=MAX_ROWS, max_beam=1)
    yield d
    d.close()


def _inputs(torch, M, d, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, d)).astype(np.float32)
    E = (rng.standard_normal((V, d)) * 0.05).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.1 * rng.standard_normal(d)).astype(np.float32)
    return [torch.tensor(a, device="cuda") for a in (x, E, g, b)]


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.gpu
def test_two_calls_match_context_op(vocab_ctx):
    """Two calls in a row, on different inputs, each against w4j_op_logits_argmax on the same
    inputs.  Same kernels and block count, so ids must be equal and log-probabilities agree to
    1e-9 (tolerance of this test)."""
    import torch

    d = 384
    for M, seed in ((5, 1), (MAX_ROWS, 2)):
        x, E, g, b = _inputs(torch, M, d, seed)
        tok_a = torch.full((M,), -7, dtype=torch.int32, device="cuda")
        lp_a = torch.zeros(M, dtype=torch.float64, device="cuda")
        tok_b, lp_b = tok_a.clone(), lp_a.clone()
        check(_call(torch.cuda.current_device(), _vp(x), M, d, _vp(E), V, _vp(g), _vp(b), _vp(tok_a), _vp(lp_a)))
        check(lib().w4j_op_logits_argmax(vocab_ctx._ctx, _vp(x), M, _vp(E), V, _vp(g), _vp(b), _vp(tok_b),
                                         _vp(lp_b), None))
        torch.cuda.synchronize()
        assert (tok_a >= 0).all()
        assert tok_a.tolist() == tok_b.tolist()
        np.testing.assert_allclose(lp_a.cpu().numpy(), lp_b.cpu().numpy(), rtol=0, atol=1e-9)


@pytest.mark.gpu
def test_no_device_memory_taken():
    """Free device memory is the same before and after repeated calls (after the first one,
    which may load the library's device code)."""
    import torch

    d, M = 384, 8
    x, E, g, b = _inputs(torch, M, d, 3)
    tok = torch.zeros(M, dtype=torch.int32, device="cuda")
    lp = torch.zeros(M, dtype=torch.float64, device="cuda")
    dev = torch.cuda.current_device()
    check(_call(dev, _vp(x), M, d, _vp(E), V, _vp(g), _vp(b), _vp(tok), _vp(lp)))
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(5):
        check(_call(dev, _vp(x), M, d, _vp(E), V, _vp(g), _vp(b), _vp(tok), _vp(lp)))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


@pytest.mark.gpu
def test_wait_timeout_reports_through_error_word(vocab_ctx):
    """A bounded wait inside the vocabulary pass that runs out (the test hook withholds the kernel's
    weight copies, so no GPU fault is involved) is reported through the error word: every id -1,
    every log-probability NaN.  The next call is normal again, which shows the word was cleared.
    The context op reports the same way through its own error word."""
    import torch

    d, M = 384, 4
    x, E, g, b = _inputs(torch, M, d, 5)
    dev = torch.cuda.current_device()
    tok = torch.zeros(M, dtype=torch.int32, device="cuda")
    lp = torch.zeros(M, dtype=torch.float64, device="cuda")
    tok_b, lp_b = tok.clone(), lp.clone()
    check(lib().w4j_test_withhold_logits_copies(1))
    try:
        check(_call(dev, _vp(x), M, d, _vp(E), V, _vp(g), _vp(b), _vp(tok), _vp(lp)))
        torch.cuda.synchronize()
    finally:
        check(lib().w4j_test_withhold_logits_copies(0))
    assert tok.tolist() == [-1] * M and bool(torch.isnan(lp).all())
    check(_call(dev, _vp(x), M, d, _vp(E), V, _vp(g), _vp(b), _vp(tok), _vp(lp)))
    check(lib().w4j_op_logits_argmax(vocab_ctx._ctx, _vp(x), M, _vp(E), V, _vp(g), _vp(b), _vp(tok_b), _vp(lp_b),
                                     None))
    torch.cuda.synchronize()
    assert (tok >= 0).all() and tok.tolist() == tok_b.tolist()
    # the context op
    check(lib().w4j_test_withhold_logits_copies(1))
    try:
        check(lib().w4j_op_logits_argmax(vocab_ctx._ctx, _vp(x), M, _vp(E), V, _vp(g), _vp(b), _vp(tok_b),
                                         _vp(lp_b), None))
        torch.cuda.synchronize()
    finally:
        check(lib().w4j_test_withhold_logits_copies(0))
    assert tok_b.tolist() == [-1] * M and bool(torch.isnan(lp_b).all())
    check(lib().w4j_op_logits_argmax(vocab_ctx._ctx, _vp(x), M, _vp(E), V, _vp(g), _vp(b), _vp(tok_b), _vp(lp_b),
                                     None))
    torch.cuda.synchronize()
    assert tok_b.tolist() == tok.tolist()
