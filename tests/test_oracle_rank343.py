"""Pin the rank-343 oracle to the reference's own rank-343 kernels.

``golden/make_golden_rank343.py`` ran ``generated/rank343_8x8x8.py`` of the
reference under the Triton interpreter.  The FP16 left and right planes must
match bit for bit (same circuit, same association).  The reference's output
side is a matrix product of the FP16 products with the +-1 coefficient
matrix, accumulated in FP32 in an order the hardware chooses, so the oracle's
ascending-order sum must agree within one FP16 ulp of the rounded result.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from inputs import digest, random_products, randn_fp16
from oracle import fmm_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
RECORD = json.loads((GOLDEN / "golden_rank343.json").read_text())
ARRAYS = np.load(GOLDEN / "golden_rank343.npz")


def _fp16(key):
    return ARRAYS[key].view(np.float16)


def _within_one_ulp(candidate, reference):
    c = np.asarray(candidate, dtype=np.float16).astype(np.float64)
    r = np.asarray(reference, dtype=np.float16).astype(np.float64)
    ulp = np.spacing(np.abs(r).astype(np.float16)).astype(np.float64)
    return np.all(np.abs(c - r) <= ulp)


@pytest.mark.parametrize("case", RECORD["cases"], ids=lambda c: "x".join(map(str, c["shape"])))
def test_rank343_oracle_matches_reference_kernels(case):
    M, K, N = case["shape"]
    A = randn_fp16((M, K), 0)
    B = randn_fp16((K, N), 1)
    assert digest(A) == case["A"] and digest(B) == case["B"], "input generation drifted"
    L = oracle.left_transform("rank343", A.float().numpy())
    R = oracle.right_transform("rank343", B.float().numpy())
    assert digest(L.view(np.int16)) == case["left"]
    assert digest(R.view(np.int16)) == case["right"]
    bm, _, bn = oracle.block_dims(M, K, N, 8)
    P = random_products(343, bm, bn, seed=3)
    assert digest(P) == case["P"]
    C = oracle.output_transform("rank343", P.numpy(), M, N, None, "fp16")
    key = f"rank343_{M}x{K}x{N}_output"
    assert _within_one_ulp(C, _fp16(key))
    # most elements agree exactly: FP32 sums of at most 64 FP16 terms
    assert np.mean(C.astype(np.float16) == _fp16(key)) > 0.99


def test_rank343_exact_integer_product():
    A = _fp16("rank343_exact_A").astype(np.float32)
    B = _fp16("rank343_exact_B").astype(np.float32)
    C = oracle.matmul("rank343", A, B)
    assert np.array_equal(C, A @ B)
    assert np.array_equal(C.astype(np.float16), _fp16("rank343_exact_C"))


def test_rank343_coefficients_are_signed_units():
    W = oracle.output_coefficients("rank343")
    assert W.shape == (64, 343)
    assert set(np.unique(W).tolist()) == {-1, 0, 1}
    assert int((W != 0).sum()) == 12 ** 3


def test_rank343_whole_product_close_to_fp64():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((40, 48)).astype(np.float16).astype(np.float32)
    B = rng.standard_normal((48, 56)).astype(np.float16).astype(np.float32)
    C = oracle.matmul("rank343", A, B)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    assert oracle.relative_l2(C, exact) < 5e-3
