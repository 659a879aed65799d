"""Pin the oracle to the reference's own numpy restatement (tools/validate_decode_steps.py).

tests/golden/make_golden.py ran the reference's load_ggml + decoder_step on seeded
synthetic models and recorded, per greedy step, the token, top-5 and the first logits;
this replays the same inputs through the oracle and applies the reference's parity
protocol (ValidateAgainstReferenceTest.java:145-161 top-5 ids, :173-255 drift < 0.03).
The only numeric difference allowed for is the f16-table GELU of the Java path
(Tensor.java:493-538) against the exact tanh GELU of the numpy script.
"""
import numpy as np
import pytest

from oracle import oracle as O
from whisper4j_b200 import ggml

from .helpers import encoder_output, load_golden, parsed


@pytest.mark.parametrize("case", ["small_rand", "tiny_en"])
def test_oracle_matches_reference_restatement(case):
    fx = load_golden(case)
    dims = ggml.ModelDimensions(**fx["dims"])
    opts = tuple(sorted(fx["synthetic_options"].items()))
    m = O.OracleModel(parsed(dims, fx["model_seed"], "f16", opts))
    xa = encoder_output(fx["xa_seed"], dims.n_audio_ctx, dims.n_text_state)
    cache = m.new_cache()
    for s in fx["steps"]:
        lg = m.forward(s["input"], xa, cache)
        last = lg[-1]
        # greedy token and top-5 ids exactly (ValidateAgainstReferenceTest.java:145)
        assert int(np.argmax(last)) == s["token"], f"step {s['step']}"
        order = np.argsort(-last, kind="stable")[:5].tolist()
        assert order == s["top5"], f"step {s['step']}"
        # drift well under the reference protocol's 0.03 (:251-253)
        np.testing.assert_allclose(last[:8], s["first8"], atol=1e-3)
        np.testing.assert_allclose(last[s["top5"]], s["top5_scores"], atol=1e-3)
        np.testing.assert_allclose(lg[0, :8], s["row0_first8"], atol=1e-3)
    assert len(cache) == len(fx["prompt"]) + len(fx["steps"]) - 1
