"""The oracle against the reference's own tensor unit tests (TensorTest.java, SimdOpsTest.java).

Each expected value is the one the reference test asserts, with the same tolerance.
"""
import numpy as np
import pytest

from oracle import oracle as O

from .helpers import SMALL, parsed


def test_matmul_2x3_times_3x2():  # TensorTest.java:10-20
    c = O.matmul([[1, 2, 3], [4, 5, 6]], [[7, 8], [9, 10], [11, 12]])
    np.testing.assert_allclose(c, [[58, 64], [139, 154]], atol=1e-4)


def test_matmul_identity():  # TensorTest.java:22-28
    a = np.array([[1, 2], [3, 4]], np.float32)
    np.testing.assert_allclose(O.matmul(a, np.eye(2)), a, atol=1e-5)


def test_matmul_transb():  # TensorTest.java:223-232
    np.testing.assert_allclose(O.matmul_transb([[1, 2], [3, 4]], [[5, 6], [7, 8]]), [[17, 23], [39, 53]], atol=1e-4)


def test_matmul_transb_non_square():  # TensorTest.java:234-244
    a = [[1, 2, 3], [4, 5, 6]]
    np.testing.assert_allclose(O.matmul_transb(a, a), [[14, 32], [32, 77]], atol=1e-4)


def test_matmul_transb_m1():  # TensorTest.java:246-256
    c = O.matmul_transb([[1, 2, 3, 4]], [[1, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0]])
    assert c.shape == (1, 3)
    np.testing.assert_allclose(c, [[1, 2, 3]], atol=1e-4)


def test_matmul_transb_scaled():  # matmulScaled semantics (TensorTest.java:258-268): alpha after the dot
    c = O.matmul_transb([[1, 2], [3, 4]], [[5, 7], [6, 8]], alpha=0.5)
    np.testing.assert_allclose(c, [[9.5, 11], [21.5, 25]], atol=1e-4)


def test_softmax():  # TensorTest.java:270-278
    np.testing.assert_allclose(O.softmax([[1, 2, 3, 4]])[0], [0.0321, 0.0871, 0.2369, 0.6439], atol=1e-3)


def test_layer_norm():  # TensorTest.java:280-290
    y = O.layer_norm([[1, 2, 3, 4, 5]], np.ones(5), np.zeros(5))[0]
    assert abs(y[0] + 1.4142) < 1e-3 and abs(y[2]) < 1e-3 and abs(y[4] - 1.4142) < 1e-3


def test_gelu_lut():  # TensorTest.java:292-301 (f16 table, tolerance 0.01)
    m = O.OracleModel(parsed(SMALL, 3))
    g = m.gelu(np.array([-2, -1, 0, 1, 2], np.float32))
    np.testing.assert_allclose(g, [-0.0454, -0.1588, 0, 0.8412, 1.9546], atol=0.01)


def test_gelu_table_is_f16_indexed():
    # Tensor.java:493-501: entry i is the tanh GELU of the f16 value with bit pattern i
    m = O.OracleModel(parsed(SMALL, 3))
    t = m.gelu_table()
    xs = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    finite = np.isfinite(xs) & (np.abs(xs) < 8)
    with np.errstate(invalid="ignore", over="ignore"):  # the NaN / inf patterns are masked out below
        ref = 0.5 * xs * (1 + np.tanh(np.float32(np.sqrt(2 / np.pi)) * (xs + np.float32(0.044715) * xs ** 3)))
    np.testing.assert_allclose(t[finite], ref[finite], atol=2e-6, rtol=2e-6)


def test_dot_scalar():  # SimdOpsTest.java:23-31
    assert O.dot([1, 2, 3, 4], [5, 6, 7, 8]) == pytest.approx(70, abs=1e-4)


def test_dot_512():  # SimdOpsTest.java:53-70
    n = 512
    a = (np.arange(n) * 0.01).astype(np.float32)
    b = ((n - np.arange(n)) * 0.01).astype(np.float32)
    exp = np.float32(0)
    for i in range(n):
        exp = np.float32(exp + a[i] * b[i])
    assert O.dot(a, b) == pytest.approx(float(exp), abs=0.1)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_f16_rounding_matches_ieee(seed):
    # Float.floatToFloat16 is IEEE round-to-nearest-even; numpy's conversion is the same rule
    rng = np.random.default_rng(seed)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10.0 ** rng.integers(-8, 5, 2000),
                        np.array([65504, 65519, 65520, 1e-8, 2.98e-8, 6e-8, -0.0, 0.0], np.float32)]).astype(np.float32)
    with np.errstate(over="ignore"):  # values past the f16 range round to infinity on purpose
        want = x.astype(np.float16).view(np.uint16)
    got = np.array([O.f32_to_f16_bits(float(v)) for v in x], np.uint16)
    np.testing.assert_array_equal(got, want)
