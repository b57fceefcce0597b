"""The CPU oracle pinned against the reference's own known answers, plus the
properties the restatement must have (no GPU needed)."""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")


def _kat():
    with open(GOLDEN) as f:
        return json.load(f)


def test_selfcheck_kat(oracle):
    assert oracle.selfcheck_kat() == 0


def test_gemm_kat_all_entries(oracle):
    g = _kat()["gemm"]
    a = np.array(g["a"], np.float32).reshape(g["m"], g["k"])
    b = np.array(g["b"], np.float32).reshape(g["k"], g["n"])
    want = np.array(g["c"], np.float32).reshape(g["m"], g["n"])
    assert np.array_equal(oracle.matmul(a, b), want)
    assert np.array_equal(oracle.gemm_avx2_restated(a, b), want)
    # gemm_dot_f32's transposed indexing: the same product through A^T / B^T views.
    assert np.array_equal(oracle.matmul(np.ascontiguousarray(a.T).T, np.ascontiguousarray(b.T).T), want)


def test_relu_kat(oracle):
    r = _kat()["relu"]
    x = np.array([float(v) for v in r["input"]], np.float32)
    y = oracle.relu(x)
    bits = y.view(np.uint32)
    assert bits[0] == np.float32(0.0).view(np.uint32)      # -4 -> +0
    assert bits[2] == np.float32(0.0).view(np.uint32)      # -0 -> +0
    assert bits[6] == np.float32(4.0).view(np.uint32)
    assert np.isnan(y[7])
    assert y[8] == np.inf and y[4] == np.float32(0.25)


NEG0 = np.float32(-0.0).view(np.uint32)
POS0 = np.float32(0.0).view(np.uint32)


def test_gelu_tanh_kat(oracle):
    r = _kat()["gelu_tanh"]
    x = np.array([float(v) for v in r["input"]], np.float32)
    y = oracle.activation(x, oracle.EPI_GELU_TANH)
    bits = y.view(np.uint32)
    assert bits[2] == NEG0 and bits[3] == POS0
    assert np.isnan(y[7]) and y[8] == np.inf


def test_gelu_erf_kat(oracle):
    r = _kat()["gelu_erf"]
    x = np.array([float(v) for v in r["input"]], np.float32)
    y = oracle.activation(x, oracle.EPI_GELU_ERF)
    assert abs(float(y[0]) + 0.00012668497) <= 1e-8
    assert abs(float(y[5]) - 0.8413448) <= 3e-7
    bits = y.view(np.uint32)
    assert bits[2] == NEG0 and bits[3] == POS0
    assert np.isnan(y[7]) and y[8] == np.inf


def _ulps(a, b):
    """Distance in f32 units in the last place (same-sign finite values)."""
    ia = a.astype(np.float32).view(np.int32).astype(np.int64)
    ib = b.astype(np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


def test_activations_against_independent_f64_formulas(oracle):
    """The restated activations stay within 1-2 f32 ulp of the same formulas
    evaluated independently in f64 (math.erf, numpy tanh / exp), over normal
    values and the range ends; special values as the reference defines them."""
    import math
    x = np.concatenate([oracle.randn(20000, 7, 3.0), np.linspace(-30, 30, 2001, dtype=np.float32)]).astype(np.float32)
    xd = x.astype(np.float64)
    erf = np.vectorize(math.erf)
    ref_gelu_erf = (0.5 * xd * (1.0 + erf(xd / math.sqrt(2.0)))).astype(np.float32)
    got = oracle.activation(x, oracle.EPI_GELU_ERF)
    ok = np.abs(xd) < 5  # beyond, 1 + erf cancels in the independent formula
    assert _ulps(got[ok], ref_gelu_erf[ok]).max() <= 1
    ref_tanh = (0.5 * xd * (1.0 + np.tanh(0.7978846 * (xd + 0.044715 * xd ** 3)))).astype(np.float32)
    got = oracle.activation(x, oracle.EPI_GELU_TANH)
    assert np.allclose(got, ref_tanh, rtol=1e-5, atol=1e-6)
    ref_silu = (xd / (1.0 + np.exp(-xd))).astype(np.float32)
    got = oracle.activation(x, oracle.EPI_SILU)
    assert np.allclose(got, ref_silu, rtol=1e-5, atol=1e-30)
    got = oracle.activation(x, oracle.EPI_RELU6)
    assert np.array_equal(got, np.clip(x, 0, 6).astype(np.float32))
    sp = np.array([-np.inf, np.inf, -0.0, np.nan, 6.0, 7.5, -40.0], np.float32)
    r6 = oracle.activation(sp, oracle.EPI_RELU6)
    assert list(r6[[0, 1, 4, 5]]) == [0.0, 6.0, 6.0, 6.0] and r6.view(np.uint32)[2] == POS0 and np.isnan(r6[3])
    si = oracle.activation(sp, oracle.EPI_SILU)
    assert si.view(np.uint32)[0] == NEG0 and si[1] == np.inf and si.view(np.uint32)[2] == NEG0 and np.isnan(si[3])
    ge = oracle.activation(sp, oracle.EPI_GELU_ERF)
    assert ge.view(np.uint32)[0] == NEG0 and ge[1] == np.inf and ge.view(np.uint32)[6] == NEG0
    with pytest.raises(ValueError):
        oracle.activation(sp, 12)


@pytest.mark.parametrize("epi", [4, 5, 6, 7, 8, 9, 10, 11])
def test_epilogue_activations(oracle, epi):
    a = oracle.randn(9 * 7, 1).reshape(9, 7)
    b = oracle.randn(7 * 6, 2).reshape(7, 6)
    bias = oracle.randn(6, 3, 0.5)
    c = oracle.matmul(a, b)
    pre = (c + bias).astype(np.float32) if epi & 1 else c
    want = oracle.activation(pre, epi)
    got = oracle.matmul(a, b, bias=bias if epi & 1 else None, epilogue=epi)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_sequential_order_is_not_reassociated(oracle):
    # 1e8 + 1 - 1e8 in increasing-p order with f32 sums gives 0, a pairwise or
    # FMA order would not: pins that every sum is a separately rounded f32 add.
    a = np.array([[1.0, 1.0, 1.0]], np.float32)
    b = np.array([[1e8], [1.0], [-1e8]], np.float32)
    assert oracle.matmul(a, b)[0, 0] == np.float32(0.0)
    # and the product is rounded before the add (no FMA): (1+2^-12)^2 - 1
    x = np.float32(1.0 + 2.0 ** -12)
    a = np.array([[x, -1.0]], np.float32)
    b = np.array([[x], [1.0]], np.float32)
    prod = np.float32(x * x)
    assert oracle.matmul(a, b)[0, 0] == np.float32(prod - np.float32(1.0))


def test_thread_count_invariance(oracle):
    a = oracle.randu(97 * 131, 11).reshape(97, 131)
    b = oracle.randu(131 * 77, 12).reshape(131, 77)
    c1 = oracle.matmul(a, b, nthreads=1)
    c8 = oracle.matmul(a, b, nthreads=8)
    assert np.array_equal(c1.view(np.uint32), c8.view(np.uint32))
    assert np.array_equal(c1.view(np.uint32), oracle.gemm_avx2_restated(a, b, nthreads=3).view(np.uint32))


def test_against_fp64(oracle):
    a = oracle.randu(256 * 512, 1).reshape(256, 512)
    b = oracle.randu(512 * 128, 2).reshape(512, 128)
    c = oracle.matmul(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.linalg.norm(c - ref) / np.linalg.norm(ref) < 2e-6
    assert np.allclose(oracle.matmul_f64(a, b), ref, rtol=1e-12, atol=1e-12)


def test_batched_broadcast_and_rows(oracle):
    a = oracle.randn(4 * 8 * 16, 5).reshape(4, 8, 16)
    b = oracle.randn(16 * 8, 6).reshape(16, 8)
    c = oracle.matmul(a, b)
    for i in range(4):
        assert np.array_equal(c[i], oracle.matmul(a[i], b))
    rows = np.array([7, 0, 3])
    cr = oracle.matmul(a[1], b, rows=rows)
    assert np.array_equal(cr, oracle.matmul(a[1], b)[rows])


def test_epilogue_bias_relu(oracle):
    a = oracle.randn(8 * 5, 1).reshape(8, 5)
    b = oracle.randn(5 * 6, 2).reshape(5, 6)
    bias = oracle.randn(6, 3, 0.1)
    c = oracle.matmul(a, b)
    want = oracle.relu((c + bias).astype(np.float32))
    got = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_k_zero_writes_positive_zero(oracle):
    a = np.zeros((3, 0), np.float32)
    b = np.zeros((0, 2), np.float32)
    c = oracle.matmul(a, b)
    assert c.shape == (3, 2) and np.all(c.view(np.uint32) == 0)


def test_rng_words_and_units(oracle):
    # SplitMix64 from seed 0: the first output is the published test value of
    # the generator (0xE220A8397B1DCDAF).
    w = oracle.splitmix64_words(0, 3)
    assert int(w[0]) == 0xE220A8397B1DCDAF
    u = oracle.randu(10000, 42, 0.0, 1.0)
    assert u.min() >= 0.0 and u.max() < 1.0
    n = oracle.randn(100001, 9)
    assert abs(float(n.mean())) < 0.02 and abs(float(n.std()) - 1.0) < 0.02


def test_numpy_generator_matches_oracle(oracle):
    from momiru_b200 import rng
    assert np.array_equal(rng.splitmix64(123, 1000), oracle.splitmix64_words(123, 1000))
    assert np.array_equal(rng.randu((333,), 5).view(np.uint32), oracle.randu(333, 5).view(np.uint32))
    assert np.array_equal(rng.randu((64,), 5, 0.0, 1.0), oracle.randu(64, 5, 0.0, 1.0))
    # Box-Muller uses libm transcendentals: equal to a few ulps, not bitwise.
    assert np.max(np.abs(rng.randn((1001,), 7, 0.02) - oracle.randn(1001, 7, 0.02))) < 1e-7
