"""Size-independent properties of the oracle (CPU): every scheme is an exact
identity over the integers, so products of small integers come out exact
through the FP32 transforms, FP64 leaf products and FP32 recombination; the
transforms are linear; and zero padding of ragged shapes is invisible."""

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import fmm_oracle as oracle

SCHEMES = ("rank7", "rank48", "rank49")


@settings(max_examples=25, deadline=None)
@given(scheme=st.sampled_from(SCHEMES), M=st.integers(1, 40), K=st.integers(1, 40),
       N=st.integers(1, 40), seed=st.integers(0, 2**31 - 1))
def test_small_integer_products_are_exact(scheme, M, K, N, seed):
    rng = np.random.default_rng(seed)
    A = rng.integers(-2, 3, (M, K)).astype(np.float32)
    W = rng.integers(-2, 3, (N, K)).astype(np.float32)
    got = oracle.linear(scheme, A, W)
    np.testing.assert_array_equal(got, A @ W.T)


@settings(max_examples=10, deadline=None)
@given(M=st.integers(1, 24), K=st.integers(1, 24), N=st.integers(1, 24), seed=st.integers(0, 2**31 - 1))
def test_rank343_small_integer_products_are_exact(M, K, N, seed):
    rng = np.random.default_rng(seed)
    A = rng.integers(-1, 2, (M, K)).astype(np.float32)
    B = rng.integers(-1, 2, (K, N)).astype(np.float32)
    np.testing.assert_array_equal(oracle.matmul("rank343", A, B), A @ B)


@settings(max_examples=20, deadline=None)
@given(scheme=st.sampled_from(SCHEMES), seed=st.integers(0, 2**31 - 1))
def test_left_transform_is_linear_on_integers(scheme, seed):
    rng = np.random.default_rng(seed)
    X = rng.integers(-4, 5, (12, 20)).astype(np.float32)
    Y = rng.integers(-4, 5, (12, 20)).astype(np.float32)
    lhs = oracle.left_transform(scheme, X + Y).astype(np.float64)
    rhs = oracle.left_transform(scheme, X).astype(np.float64) + oracle.left_transform(scheme, Y)
    np.testing.assert_array_equal(lhs, rhs)


def test_padding_rows_and_columns_do_not_change_the_result():
    rng = np.random.default_rng(3)
    A = rng.integers(-2, 3, (13, 9)).astype(np.float32)
    W = rng.integers(-2, 3, (11, 9)).astype(np.float32)
    for scheme in SCHEMES:
        s = oracle.scheme_circuits(scheme)[0]
        Ap = np.zeros((16, 12), np.float32)
        Ap[:13, :9] = A
        Wp = np.zeros((12, 12), np.float32)
        Wp[:11, :9] = W
        np.testing.assert_array_equal(oracle.linear(scheme, A, W), oracle.linear(scheme, Ap, Wp)[:13, :11])
        assert 16 % s == 0 and 12 % s == 0
