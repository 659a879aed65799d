"""Decoder token loop on the GPU against the CPU oracle (restatement of WhisperDecoder.java).

Logits: max-abs 2e-2 and relative 1e-2; token ids identical except where the oracle's
gap between the two candidates is below that tolerance (random-init weights make near
ties common), in which case the comparison stops at that step.
"""
import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml
from whisper4j_b200.decoder import WhisperDecoder

from .helpers import (LOGIT_ATOL, SMALL, SMALL_OPTS, assert_logits_close, check_beam, encoder_output,
                      first_divergence, load_golden, parsed)

pytestmark = pytest.mark.gpu

SO = tuple(sorted(SMALL_OPTS.items()))
TINY = ggml.ARCHS["tiny.en"]


@pytest.fixture(scope="module")
def small():
    gm = parsed(SMALL, 101, "f16", SO)
    d = WhisperDecoder(gm, max_streams=4, max_beam=5)
    o = O.OracleModel(gm)
    xas = [encoder_output(200 + i, SMALL.n_audio_ctx, SMALL.n_text_state) for i in range(4)]
    for i, xa in enumerate(xas):
        d.set_encoder_output(xa, slot=i)
    yield d, o, xas
    d.close()


@pytest.fixture(scope="module")
def tiny():
    gm = parsed(TINY, 21)
    d = WhisperDecoder(gm, max_streams=2, max_beam=3)
    o = O.OracleModel(gm)
    xa = encoder_output(22, TINY.n_audio_ctx, TINY.n_text_state)
    d.set_encoder_output(xa, slot=0)
    yield d, o, xa
    d.close()


def check_tokens(dec_tokens, ora_tokens, oracle, xa, prompt, masks_fn=None):
    """Equal ids, or a divergence at a near tie of the oracle's (masked) logits."""
    i = first_divergence(dec_tokens, ora_tokens)
    if i is None:
        return
    assert i < min(len(dec_tokens), len(ora_tokens)), "lengths differ without a token difference"
    cache = oracle.new_cache()
    lg = oracle.forward(list(prompt) + list(ora_tokens[:i]), xa, cache)[-1]
    if masks_fn:
        lg = masks_fn(lg, ora_tokens[:i], i)
    a, b = dec_tokens[i], ora_tokens[i]
    assert abs(float(lg[a]) - float(lg[b])) < LOGIT_ATOL, f"step {i}: {a} vs {b} gap {lg[b] - lg[a]}"


# ---------------------------------------------------------------------------
# forward (teacher forced) — WhisperDecoder.forward
# ---------------------------------------------------------------------------
def test_forward_prompt_and_steps_match_oracle(small):
    dec, ora, xas = small
    cache_d = dec.new_cache(0)
    cache_o = ora.new_cache()
    prompt = [996, 997, 998, 999]
    got = dec.forward(prompt, kv_cache=cache_d)
    want = ora.forward(prompt, xas[0], cache_o)
    assert_logits_close(got, want)
    rng = np.random.default_rng(0)
    for _ in range(12):
        t = [int(rng.integers(0, SMALL.n_vocab))]
        assert_logits_close(dec.forward(t, kv_cache=cache_d), ora.forward(t, xas[0], cache_o))


def test_forward_without_cache_leaves_cache_alone(small):
    dec, ora, xas = small
    cache = dec.new_cache(1)
    a = dec.forward([5, 6], kv_cache=cache)
    b = dec.forward([7], kv_cache=None, slot=1)  # kvCache == null (detectLanguage)
    assert_logits_close(b, ora.forward([7], xas[1], None))
    c = dec.forward([8], kv_cache=cache)
    o_cache = ora.new_cache()
    ora.forward([5, 6], xas[1], o_cache)
    assert_logits_close(c, ora.forward([8], xas[1], o_cache))
    assert_logits_close(a, ora.forward([5, 6], xas[1], None))


def test_forward_past_n_text_ctx_matches_oracle(small):
    """WhisperDecoder.java:72: offset = min(cache length, n_ctx - seqLen) while the cache keeps
    growing, so positions past n_text_ctx reuse the last positional row."""
    dec, ora, xas = small
    cache_d, cache_o = dec.new_cache(2), ora.new_cache()
    prompt = [996, 997, 998, 999]
    assert_logits_close(dec.forward(prompt, kv_cache=cache_d), ora.forward(prompt, xas[2], cache_o))
    rng = np.random.default_rng(3)
    for i in range(SMALL.n_text_ctx + 8):
        t = [int(rng.integers(0, SMALL.n_vocab))]
        assert_logits_close(dec.forward(t, kv_cache=cache_d), ora.forward(t, xas[2], cache_o),
                            what=f"position {len(prompt) + i}")
    assert len(cache_o) == len(prompt) + SMALL.n_text_ctx + 8


def test_forward_multi_token_on_filled_cache(small):
    """MultiHeadAttention.java:84-88 with Tensor.java:622-640: a multi-token call applies the
    (n_ctx x n_ctx) causal mask from key column 0 even when the cache already holds rows, so query t
    attends keys [0, t] and [n_ctx, kv_len) — not its own new rows.  Also a call that crosses
    n_text_ctx (clamped offset) and one of n_text_ctx tokens."""
    dec, ora, xas = small
    rng = np.random.default_rng(9)
    cache_d, cache_o = dec.new_cache(3), ora.new_cache()
    for n in (4, 3, 1, 20, 30, 10, 2):
        t = [int(v) for v in rng.integers(0, SMALL.n_vocab, n)]
        assert_logits_close(dec.forward(t, kv_cache=cache_d), ora.forward(t, xas[3], cache_o),
                            what=f"{n} tokens after {len(cache_o) - n}")
    full = [int(v) for v in rng.integers(0, SMALL.n_vocab, SMALL.n_text_ctx)]
    cache_d, cache_o = dec.new_cache(3), ora.new_cache()
    assert_logits_close(dec.forward(full, kv_cache=cache_d), ora.forward(full, xas[3], cache_o))
    assert_logits_close(dec.forward(full[:40], kv_cache=cache_d), ora.forward(full[:40], xas[3], cache_o))
    assert_logits_close(dec.forward(full[:40], kv_cache=None, slot=3), ora.forward(full[:40], xas[3], None))
    with pytest.raises(ValueError):
        dec.forward([1] * (SMALL.n_text_ctx + 1), kv_cache=cache_d)


def test_beam_past_n_text_ctx_matches_oracle(small):
    dec, ora, xas = small
    prompt, eot, n = [996, 997], 995, SMALL.n_text_ctx + 6
    r = dec.decode_beam(None, prompt, eot, n, suppress_tokens=[eot], beam_size=3)
    w = ora.decode_beam(xas[0], prompt, eot, n, suppress=[eot], beam=3, trace=True)
    assert len(r.tokens) == n
    check_beam(r.tokens, w, ora, xas[0], prompt, [eot], eot, 3, n)


@pytest.mark.parametrize("case", ["small_rand", "tiny_en"])
def test_forward_matches_reference_golden(case):
    """The device path against the reference's own numpy restatement (golden fixtures)."""
    fx = load_golden(case)
    dims = ggml.ModelDimensions(**fx["dims"])
    gm = parsed(dims, fx["model_seed"], "f16", tuple(sorted(fx["synthetic_options"].items())))
    xa = encoder_output(fx["xa_seed"], dims.n_audio_ctx, dims.n_text_state)
    with WhisperDecoder(gm, max_streams=1, max_beam=1) as dec:
        dec.set_encoder_output(xa, 0)
        cache = dec.new_cache(0)
        for s in fx["steps"]:
            lg = dec.forward(s["input"], kv_cache=cache)
            last = lg[-1]
            assert np.abs(last[:8] - np.array(s["first8"])).max() < 0.03  # ValidateAgainstReferenceTest drift
            assert np.abs(last[s["top5"]] - np.array(s["top5_scores"])).max() < LOGIT_ATOL
            top = s["top5_scores"]
            if top[0] - top[1] > LOGIT_ATOL:
                assert int(np.argmax(last)) == s["token"]


def test_forward_tiny_full_vocab(tiny):
    dec, ora, xa = tiny
    cache_d, cache_o = dec.new_cache(0), ora.new_cache()
    prompt = [50257, 50258, 50259, 50362]
    assert_logits_close(dec.forward(prompt, kv_cache=cache_d), ora.forward(prompt, xa, cache_o))
    for t in (400, 1000, 50000, 7):
        assert_logits_close(dec.forward([t], kv_cache=cache_d), ora.forward([t], xa, cache_o))


# ---------------------------------------------------------------------------
# greedy — WhisperDecoder.decode
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("slot", [0, 2])
def test_greedy_forced_length_matches_oracle(small, slot):
    dec, ora, xas = small
    prompt, eot = [996, 997, 998, 999], 995
    r = dec.decode_batch([slot], [prompt], eot, 40, suppress_tokens=[eot], no_speech_token=3)[0]
    w = ora.decode(xas[slot], prompt, eot, 40, suppress=[eot], no_speech=3)
    check_tokens(r.tokens, w["tokens"], ora, xas[slot], prompt)
    if r.tokens == w["tokens"]:
        assert len(r.tokens) == 40
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2 + 1e-3 * abs(w["sum_logprob"]))
        assert r.avg_logprob == pytest.approx(w["avg_logprob"], abs=1e-3)
    assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)


def test_greedy_stops_at_eot(small):
    dec, ora, xas = small
    prompt = [996, 997, 998, 999]
    free = ora.decode(xas[0], prompt, 995, 20, suppress=[995])
    eot = free["tokens"][5]  # make the 6th greedy choice the end-of-text id
    r = dec.decode(None, prompt, eot, 20)
    w = ora.decode(xas[0], prompt, eot, 20)
    check_tokens(r.tokens, w["tokens"], ora, xas[0], prompt)
    if r.tokens == w["tokens"]:
        assert len(r.tokens) < 20 and eot not in r.tokens


def test_greedy_batch_equals_single(small):
    dec, ora, xas = small
    prompts = [[996, 997, 998, 999], [996, 997, 998, 10], [996, 997, 11, 12]]
    batch = dec.decode_batch([0, 1, 3], prompts, 995, 24, suppress_tokens=[995])
    for (slot, p), rb in zip(zip([0, 1, 3], prompts), batch):
        rs = dec.decode_batch([slot], [p], 995, 24, suppress_tokens=[995])[0]
        assert rb.tokens == rs.tokens
        assert rb.sum_logprob == pytest.approx(rs.sum_logprob, abs=1e-9)
        w = ora.decode(xas[slot], p, 995, 24, suppress=[995])
        check_tokens(rb.tokens, w["tokens"], ora, xas[slot], p)


def test_greedy_suppress_and_timestamps(small):
    dec, ora, xas = small
    prompt, eot, tb = [996, 997, 998, 999], 900, 901
    sup = [eot, 3, 5, 7, 11]
    r = dec.decode(None, prompt, eot, 30, suppress_tokens=sup, timestamp_begin=tb)
    w = ora.decode(xas[0], prompt, eot, 30, suppress=sup, ts_begin=tb)
    check_tokens(r.tokens, w["tokens"], ora, xas[0], prompt)
    assert r.tokens[0] >= tb  # first token is forced to be a timestamp


def test_greedy_max_tokens_edge_cases(small):
    dec, ora, xas = small
    r0 = dec.decode(None, [996], 995, 0)
    assert r0.tokens == [] and r0.avg_logprob == 0.0
    r1 = dec.decode(None, [996], 995, 1, suppress_tokens=[995])
    w1 = ora.decode(xas[0], [996], 995, 1, suppress=[995])
    check_tokens(r1.tokens, w1["tokens"], ora, xas[0], [996])
    # prompt + generated fills the whole 64-position context
    rf = dec.decode(None, [996, 997], 995, SMALL.n_text_ctx - 1, suppress_tokens=[995])
    assert len(rf.tokens) == SMALL.n_text_ctx - 1
    # past n_text_ctx the reference reuses the last positional row while its cache keeps growing
    # (WhisperDecoder.java:72): same as the oracle
    n = SMALL.n_text_ctx + 12
    rp = dec.decode(None, [996, 997], 995, n, suppress_tokens=[995])
    wp = ora.decode(xas[0], [996, 997], 995, n, suppress=[995])
    assert len(rp.tokens) == n
    check_tokens(rp.tokens, wp["tokens"], ora, xas[0], [996, 997])
    with pytest.raises(ValueError):
        dec.decode(None, [996] * (SMALL.n_text_ctx + 1), 995, 4)  # a prompt longer than the positional table


def test_tiny_greedy_64_tokens(tiny):
    dec, ora, xa = tiny
    prompt, eot = [50257, 50258, 50259, 50362], 50256
    r = dec.decode(None, prompt, eot, 64, suppress_tokens=[eot], no_speech_token=50361)
    w = ora.decode(xa, prompt, eot, 64, suppress=[eot], no_speech=50361)
    check_tokens(r.tokens, w["tokens"], ora, xa, prompt)
    assert len(r.tokens) == 64
    assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-7)


# ---------------------------------------------------------------------------
# beam search — WhisperDecoder.decodeBeam
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("beam", [2, 3, 5])
def test_beam_forced_length_matches_oracle(small, beam):
    dec, ora, xas = small
    prompt, eot = [996, 997, 998, 999], 995
    r = dec.decode_beam_batch([1], [prompt], eot, 16, suppress_tokens=[eot], no_speech_token=3, beam_size=beam)[0]
    w = ora.decode_beam(xas[1], prompt, eot, 16, suppress=[eot], no_speech=3, beam=beam, trace=True)
    if check_beam(r.tokens, w, ora, xas[1], prompt, [eot], eot, beam, 16) == "equal":
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)
    assert len(r.tokens) == 16
    assert r.no_speech_prob == pytest.approx(w["no_speech_prob"], rel=2e-2, abs=1e-6)


def test_beam_with_finished_sequences(small):
    dec, ora, xas = small
    prompt = [996, 997, 998, 999]
    free = ora.decode_beam(xas[2], prompt, 995, 12, suppress=[995], beam=3)
    eot = free["tokens"][4]  # an id the beams actually reach, so sequences finish early
    r = dec.decode_beam_batch([2], [prompt], eot, 12, beam_size=3)[0]
    w = ora.decode_beam(xas[2], prompt, eot, 12, beam=3, trace=True)
    if check_beam(r.tokens, w, ora, xas[2], prompt, [], eot, 3, 12) == "equal":
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)


def test_beam_batch_equals_single(small):
    dec, ora, xas = small
    prompts = [[996, 997, 998, 999], [996, 997, 998, 20]]
    batch = dec.decode_beam_batch([0, 3], prompts, 995, 10, suppress_tokens=[995], beam_size=4)
    for slot, p, rb in zip([0, 3], prompts, batch):
        rs = dec.decode_beam_batch([slot], [p], 995, 10, suppress_tokens=[995], beam_size=4)[0]
        assert rb.tokens == rs.tokens


def test_tiny_beam(tiny):
    dec, ora, xa = tiny
    prompt, eot = [50257, 50258, 50259, 50362], 50256
    r = dec.decode_beam(None, prompt, eot, 12, suppress_tokens=[eot], beam_size=3)
    w = ora.decode_beam(xa, prompt, eot, 12, suppress=[eot], beam=3, trace=True)
    if check_beam(r.tokens, w, ora, xa, prompt, [eot], eot, 3, 12) == "equal":
        assert r.sum_logprob == pytest.approx(w["sum_logprob"], abs=2e-2)
    assert len(r.tokens) == 12


# ---------------------------------------------------------------------------
# Q8_0 weights (GgmlLoader.java:292-300)
# ---------------------------------------------------------------------------
def test_q8_0_model_matches_oracle():
    gm = parsed(SMALL, 77, "q8_0", SO)
    ora = O.OracleModel(gm)
    xa = encoder_output(78, SMALL.n_audio_ctx, SMALL.n_text_state)
    with WhisperDecoder(gm, max_streams=1, max_beam=2) as dec:
        dec.set_encoder_output(xa, 0)
        cache_d, cache_o = dec.new_cache(0), ora.new_cache()
        prompt = [996, 997, 998, 999]
        assert_logits_close(dec.forward(prompt, kv_cache=cache_d), ora.forward(prompt, xa, cache_o))
        r = dec.decode(None, prompt, 995, 20, suppress_tokens=[995])
        w = ora.decode(xa, prompt, 995, 20, suppress=[995])
        check_tokens(r.tokens, w["tokens"], ora, xa, prompt)
        rb = dec.decode_beam(None, prompt, 995, 8, suppress_tokens=[995], beam_size=2)
        wb = ora.decode_beam(xa, prompt, 995, 8, suppress=[995], beam=2, trace=True)
        if check_beam(rb.tokens, wb, ora, xa, prompt, [995], 995, 2, 8) == "equal":
            assert rb.sum_logprob == pytest.approx(wb["sum_logprob"], abs=2e-2)


# ---------------------------------------------------------------------------
# sampling and the fallback policy
# ---------------------------------------------------------------------------
def test_sampling_is_seeded_and_valid(small):
    dec, _, _ = small
    prompt = [996, 997, 998, 999]
    a = dec.decode(None, prompt, 995, 16, suppress_tokens=[995, 4], temperature=0.8, seed=7)
    b = dec.decode(None, prompt, 995, 16, suppress_tokens=[995, 4], temperature=0.8, seed=7)
    c = dec.decode(None, prompt, 995, 16, suppress_tokens=[995, 4], temperature=0.8, seed=8)
    assert a.tokens == b.tokens and len(a.tokens) == 16
    assert 4 not in a.tokens and 995 not in a.tokens
    assert a.tokens != c.tokens
    assert np.isfinite(a.avg_logprob)


@pytest.mark.parametrize("allowed,n,seed", [(None, 24, 3), (8, 100, 11)])
def test_decode_with_fallback_matches_policy(small, allowed, n, seed):
    """w4j_decode_with_fallback against a restatement of WhisperDecoder.java:119-149 driven by the same
    device decodes (each temperature decoded alone with the same seed; sampling is seeded, so the
    attempts are reproducible).  Random-init log-probabilities are far below -1, so every result
    needs a fallback: with the full vocabulary the temperature-0 result compresses below 2.4 and the
    policy stops there (it must also match the oracle); with 8 allowed ids over 100 forced tokens the
    greedy ids compress above 2.4 and the policy goes on to the sampled attempts."""
    from .helpers import fallback_policy_ref
    dec, ora, xas = small
    prompt = [996, 997, 998, 999]
    sup = [995] if allowed is None else [t for t in range(SMALL.n_vocab) if not 100 <= t < 100 + allowed]
    r = dec.decode_with_fallback(None, prompt, 995, n, suppress_tokens=sup, seed=seed)
    want, want_t, attempts = fallback_policy_ref(
        lambda t: dec.decode(None, prompt, 995, n, suppress_tokens=sup, temperature=t, seed=seed))
    assert r.temperature == want_t and r.tokens == want.tokens
    assert r.avg_logprob == pytest.approx(want.avg_logprob, abs=1e-6)
    if allowed is None:
        assert attempts == 1 and r.temperature == 0.0
        w = ora.decode(xas[0], prompt, 995, n, suppress=sup)
        check_tokens(r.tokens, w["tokens"], ora, xas[0], prompt)
    assert len(r.tokens) == n


def test_cancel_from_another_thread(small):
    """w4j_cancel (TranscriptionHandle cancellation, WhisperModel.java:620-633) from a second host thread
    stops a long decode at a step boundary with W4J_ERR_CANCELLED; the context stays usable."""
    import threading
    import time

    from whisper4j_b200._lib import CancelledError
    dec, ora, xas = small
    prompt = [996, 997, 998, 999]
    done = threading.Event()

    def canceller():
        while not done.is_set():
            dec.cancel()
            time.sleep(0.0005)

    th = threading.Thread(target=canceller)
    th.start()
    try:
        with pytest.raises(CancelledError):
            dec.decode(None, prompt, 995, 4000, suppress_tokens=[995])
    finally:
        done.set()
        th.join()
    r = dec.decode(None, prompt, 995, 16, suppress_tokens=[995])
    w = ora.decode(xas[0], prompt, 995, 16, suppress=[995])
    check_tokens(r.tokens, w["tokens"], ora, xas[0], prompt)


def test_host_injected_failures(small):
    """Failures made on the host, none on the GPU: a context whose caches cannot be allocated
    (W4J_ERR_OOM -> MemoryError), a truncated GGML payload (IllegalArgumentException -> ValueError);
    the existing context keeps working afterwards."""
    from whisper4j_b200._lib import Dims, check, lib
    import ctypes
    dec, ora, xas = small
    gm = parsed(SMALL, 101, "f16", SO)
    big = ggml.ModelDimensions(80, 1500, 1280, 20, 1, 51866, 448, 1280, 20, 4)
    cd = Dims(*[getattr(big, f) for f in ("n_mels", "n_audio_ctx", "n_audio_state", "n_audio_head", "n_audio_layer",
                                           "n_vocab", "n_text_ctx", "n_text_state", "n_text_head", "n_text_layer")])
    h = ctypes.c_void_p()
    with pytest.raises(MemoryError):  # 1e5 streams x 31 MB of cross K/V: far beyond any GPU
        check(lib().w4j_ctx_create(ctypes.byref(cd), 0, 100000, 1, ctypes.byref(h)))
    assert not h.value
    t = gm.tensors["decoder.blocks.0.mlp.0.weight"]
    buf = np.frombuffer(t.data, np.uint8)[:-2]  # two bytes short
    ne = (ctypes.c_int64 * len(t.ne))(*t.ne)
    with pytest.raises(ValueError, match="payload size"):
        check(lib().w4j_upload_tensor(dec._ctx, t.name.encode(), t.ttype, ne, len(t.ne),
                                      buf.ctypes.data_as(ctypes.c_void_p), buf.size))
    r = dec.decode(None, [996, 997, 998, 999], 995, 8, suppress_tokens=[995])
    assert len(r.tokens) == 8


# ---------------------------------------------------------------------------
# errors (IllegalArgumentException / IllegalStateException in the reference)
# ---------------------------------------------------------------------------
def test_errors(small):
    from whisper4j_b200._lib import IllegalStateError
    dec, _, _ = small
    with pytest.raises(ValueError):
        dec.decode(None, [SMALL.n_vocab], 995, 4)  # token id out of range
    with pytest.raises(ValueError):
        dec.decode(None, [996], SMALL.n_vocab + 3, 4)  # eot out of range
    with pytest.raises(ValueError):
        dec.decode_beam(None, [996], 995, 4, beam_size=6)  # beyond the context's max_beam
    with pytest.raises(ValueError):
        dec.decode_batch([0, 0], [[996], [996]], 995, 4)  # same stream twice
    gm = parsed(SMALL, 101, "f16", SO)
    with WhisperDecoder(gm, max_streams=2, max_beam=1) as d2:
        with pytest.raises(IllegalStateError):
            d2.decode_batch([1], [[996]], 995, 4)  # no encoder output for the slot
    partial = ggml.GgmlModel(gm.dims, gm.ftype, gm.mel_filters, gm.vocab,
                             {k: v for k, v in gm.tensors.items() if "mlp.2.bias" not in k})
    with pytest.raises(IllegalStateError, match="weight not found"):
        WhisperDecoder(partial, max_streams=1, max_beam=1)
