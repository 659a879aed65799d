"""Single kernels of the decode step through the C ABI, against fp32 references of the same op.

w4j_op_linear = [LayerNorm] -> Linear -> [GELU | residual] (nn/Linear.java:23-26, nn/LayerNorm.java:28-30,
Tensor.geluInPlace Tensor.java:524-538, addInPlace :251-263); w4j_op_logits_argmax = final LayerNorm,
tied-embedding logits, argmax and log-softmax (WhisperDecoder.java:102-103, :566-574, :614-626).
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200._lib import GGML_F16, GGML_Q8_0, check, lib
from whisper4j_b200.decoder import WhisperDecoder

from .helpers import SMALL, SMALL_OPTS, parsed

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dec():
    d = WhisperDecoder(parsed(SMALL, 41, "f16", tuple(sorted(SMALL_OPTS.items()))), max_streams=8, max_beam=1)
    yield d
    d.close()


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


def ln_ref(x, g, b):
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + 1e-5) * g + b


def gelu_table():
    xs = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    with np.errstate(all="ignore"):
        return (0.5 * xs * (1 + np.tanh(np.float32(np.sqrt(2 / np.pi)) * (xs + np.float32(0.044715) * xs ** 3))))


# M >= 16 runs on the tcgen05 projection kernel (f16 hi/lo activations, split K over a cluster)
@pytest.mark.parametrize("M,K,N", [(1, 384, 1152), (5, 512, 512), (3, 1280, 5120), (8, 2048, 512), (16, 768, 300),
                                   (17, 512, 1536), (32, 1280, 3840), (32, 5120, 1280), (64, 1024, 4096),
                                   (64, 5120, 1280), (100, 384, 1152), (128, 512, 512), (129, 1280, 3840),
                                   (256, 1280, 5120), (256, 5120, 1280), (200, 768, 768)])
@pytest.mark.parametrize("epi", [0, 1, 2])
@pytest.mark.parametrize("use_ln", [False, True])
def test_linear_f16(dec, M, K, N, epi, use_ln):
    """Past 128 rows the tcgen05 kernel walks 128-row chunks of the activations (grid z)."""
    rng = np.random.default_rng(M * 7 + K + N + epi)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(K)).astype(np.float32)
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    dev = "cuda"
    tx, tW, tb = torch.tensor(x, device=dev), torch.tensor(W, device=dev), torch.tensor(b, device=dev)
    tg, tbeta, ty = torch.tensor(g, device=dev), torch.tensor(beta, device=dev), torch.tensor(y0, device=dev)
    check(lib().w4j_op_linear(dec._ctx, vp(tx), M, K, vp(tW), GGML_F16, N, vp(tb),
                              vp(tg) if use_ln else None, vp(tbeta) if use_ln else None, epi, vp(ty), None))
    torch.cuda.synchronize()
    xin = ln_ref(x.astype(np.float64), g, beta) if use_ln else x.astype(np.float64)
    ref = xin @ W.astype(np.float64).T + b
    if epi == 1:
        ref = gelu_table()[ref.astype(np.float32).astype(np.float16).view(np.uint16)]
    elif epi == 2:
        ref = y0 + ref
    got = ty.cpu().numpy()
    np.testing.assert_allclose(got, ref, atol=2e-4 * np.sqrt(K) + 1e-3 * (epi == 1), rtol=1e-4)


# M >= 16 with N a multiple of 128 runs on the tcgen05 kernel: int8 tiles by TMA, dequantised in
# shared memory into f16 hi / lo tiles (exact q * scale), two MMAs per k-step
@pytest.mark.parametrize("M,K,N", [(1, 512, 512), (5, 384, 1536), (2, 1280, 700), (16, 512, 512), (40, 1280, 3840),
                                   (40, 5120, 1280), (40, 1280, 5120), (129, 1280, 1280), (256, 1280, 3840),
                                   (24, 1280, 700)])
@pytest.mark.parametrize("use_ln,epi", [(False, 0), (True, 1), (False, 2)])
def test_linear_q8_0(dec, M, K, N, use_ln, epi):
    rng = np.random.default_rng(K + N + M)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    blocks = np.frombuffer(ggml.quantize_q8_0(W), np.uint8)
    Wq = ggml.dequantize(ggml.GgmlTensor("w", ggml.GGML_TYPE_Q8_0, (K, N), memoryview(blocks.tobytes())))
    tsrc = torch.tensor(blocks, device="cuda")
    tdst = torch.zeros(N * K + N * K // 16, dtype=torch.uint8, device="cuda")
    check(lib().w4j_q8_0_repack(vp(tsrc), N, K, vp(tdst), None))
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(K)).astype(np.float32)
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    tx, tb = torch.tensor(x, device="cuda"), torch.tensor(b, device="cuda")
    tg, tbeta, ty = torch.tensor(g, device="cuda"), torch.tensor(beta, device="cuda"), torch.tensor(y0, device="cuda")
    check(lib().w4j_op_linear(dec._ctx, vp(tx), M, K, vp(tdst), GGML_Q8_0, N, vp(tb), vp(tg) if use_ln else None,
                              vp(tbeta) if use_ln else None, epi, vp(ty), None))
    torch.cuda.synchronize()
    xin = ln_ref(x.astype(np.float64), g, beta) if use_ln else x.astype(np.float64)
    ref = xin @ Wq.astype(np.float64).T + b
    if epi == 1:
        ref = gelu_table()[ref.astype(np.float32).astype(np.float16).view(np.uint16)]
    elif epi == 2:
        ref = y0 + ref
    np.testing.assert_allclose(ty.cpu().numpy(), ref, atol=2e-4 * np.sqrt(K) + 1e-3 * (epi == 1), rtol=1e-4)


def test_linear_rejects_bad_shapes(dec):
    with pytest.raises(ValueError):
        check(lib().w4j_op_linear(dec._ctx, ctypes.c_void_p(16), 0, 64, ctypes.c_void_p(16), GGML_F16, 8, None,
                                  None, None, 0, ctypes.c_void_p(16), None))
    with pytest.raises(ValueError):
        check(lib().w4j_op_linear(dec._ctx, ctypes.c_void_p(16), 1, 60, ctypes.c_void_p(16), GGML_F16, 8, None,
                                  None, None, 0, ctypes.c_void_p(16), None))


def check_logits_argmax(ctx, M, d, V, seed):
    """LN -> E^T logits -> argmax + log-softmax of each row against the oracle (f32 LN, f32 GEMM).

    Tolerances: the tensor-core path rounds the normalised activations to f16 before the
    product (relative 2^-11), so two logits may swap only at a near tie (< 2e-2 apart) and
    log-probabilities agree to 2e-3."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, d)).astype(np.float32)
    E = (rng.standard_normal((V, d)) * 0.05).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.1 * rng.standard_normal(d)).astype(np.float32)
    tx, tE, tg, tb = (torch.tensor(a, device="cuda") for a in (x, E, g, b))
    tok = torch.zeros(M, dtype=torch.int32, device="cuda")
    lp = torch.zeros(M, dtype=torch.float64, device="cuda")
    check(lib().w4j_op_logits_argmax(ctx, vp(tx), M, vp(tE), V, vp(tg), vp(tb), vp(tok), vp(lp), None))
    torch.cuda.synchronize()
    ln = O.layer_norm(x, g, b)
    logits = O.matmul_transb(ln, E.astype(np.float32))
    for m in range(M):
        row = logits[m].astype(np.float64)
        want = int(np.argmax(row))
        got = int(tok[m])
        srt = np.sort(row)[::-1]
        if got != want:  # allowed only at a near tie
            assert abs(row[got] - row[want]) < 2e-2, (m, got, want)
        lse = srt[0] + np.log(np.exp(row - srt[0]).sum())
        assert float(lp[m]) == pytest.approx(row[got] - lse, abs=2e-3), m


@pytest.mark.parametrize("M", [1, 3, 5])
def test_logits_argmax_matches_oracle(dec, M):
    check_logits_argmax(dec._ctx, M, SMALL.n_text_state, SMALL.n_vocab, M)


@pytest.fixture(scope="module", params=[384, 1280], ids=["d384", "d1280"])
def vocab_dec(request):
    """A one-layer model with a full Whisper vocabulary: every logits block owns several
    128-row tiles, and up to 64 rows are live (more than 32: one tcgen05 pass per 32-row chunk)."""
    d = request.param
    dims = ggml.ModelDimensions(80, 16, d, d // 64, 1, 51864, 16, d, d // 64, 1)
    dd = WhisperDecoder(ggml.parse(ggml.synthetic_model_bytes(dims, 5)), max_streams=64, max_beam=1)
    yield dd
    dd.close()


@pytest.mark.parametrize("M", [1, 2, 3, 8, 17, 32, 40, 64])
def test_logits_argmax_full_vocab(vocab_dec, M):
    check_logits_argmax(vocab_dec._ctx, M, vocab_dec.dims.n_text_state, 51864, 100 + M)
