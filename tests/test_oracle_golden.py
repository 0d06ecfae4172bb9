"""Pin the CPU oracle to the reference's own kernels.

The fixtures in ``tests/golden`` were produced by running the reference's
generated Triton kernels (``make_golden.py``); the oracle must reproduce every
FP16 transform plane and every BF16 output bit for bit.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from inputs import digest, f32, make_linear_inputs, random_products
from oracle import fmm_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
RECORD = json.loads((GOLDEN / "golden.json").read_text())
SMALL = np.load(GOLDEN / "golden_small.npz")


def _case_id(case):
    return f"{case['scheme']}-{'x'.join(map(str, case['shape']))}"


@pytest.mark.parametrize("case", RECORD["cases"], ids=_case_id)
def test_oracle_matches_reference_kernels(case):
    name = case["scheme"]
    M, K, N = case["shape"]
    A, W, bias = make_linear_inputs(M, K, N, seed=case["seed"], bias=True)
    assert digest(A) == case["inputs"]["A"], "input generation drifted"
    assert digest(W) == case["inputs"]["W"]
    assert digest(bias) == case["inputs"]["bias"]
    L = oracle.left_transform(name, f32(A))
    R = oracle.weight_transform(name, f32(W))
    assert digest(L.view(np.int16)) == case["left"]
    assert digest(R.view(np.int16)) == case["weight"]
    s, rank = oracle.scheme_circuits(name)[:2]
    bm, _, bn = oracle.block_dims(M, K, N, s)
    P = random_products(rank, bm, bn, seed=case["product_seed"])
    assert digest(P) == case["inputs"]["P"]
    C = oracle.output_transform(name, P.numpy(), M, N)
    Cb = oracle.output_transform(name, P.numpy(), M, N, f32(bias))
    assert digest(oracle.bf16_bits(C)) == case["output"]
    assert digest(oracle.bf16_bits(Cb)) == case["output_bias"]
    key = f"{name}_{M}x{K}x{N}"
    if key + "_left" in SMALL:
        np.testing.assert_array_equal(L.view(np.int16), SMALL[key + "_left"])
        np.testing.assert_array_equal(R.view(np.int16), SMALL[key + "_weight"])
        np.testing.assert_array_equal(oracle.bf16_bits(Cb).view(np.int16), SMALL[key + "_output_bias"])


@pytest.mark.parametrize("name", ["rank7", "rank48", "rank49"])
def test_oracle_exact_integer_product(name):
    """Integer inputs in {-2..2}: the reduced-rank product is exact."""
    A = oracle.from_bf16_bits(SMALL[f"{name}_exact_A"].view(np.uint16))
    W = oracle.from_bf16_bits(SMALL[f"{name}_exact_W"].view(np.uint16))
    C = oracle.linear(name, A, W)
    np.testing.assert_array_equal(oracle.bf16_bits(C).view(np.int16), SMALL[f"{name}_exact_C"])
    np.testing.assert_array_equal(C, oracle.bf16_round((A.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)))


def test_bf16_rounding_matches_torch():
    import torch

    x = torch.randn(4096, generator=torch.Generator().manual_seed(5)) * 1e3
    x = torch.cat([x, torch.tensor([0.0, -0.0, 65504.0, 3.0e38, float("inf"), -float("inf")])])
    np.testing.assert_array_equal(
        oracle.bf16_bits(oracle.bf16_round(x.numpy())).view(np.int16),
        x.to(torch.bfloat16).view(torch.int16).numpy(),
    )


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -1.0 - 2**-8, 3.0e38, np.inf], dtype=np.float32)
    got = oracle.bf16_round(x)
    np.testing.assert_array_equal(got[:4], np.array([1.0, 1.0, 1.0 + 2**-6, -1.0], dtype=np.float32))
    assert np.isfinite(got[4]) and abs(got[4] - 3.0e38) <= 3.0e38 * 2**-8
    assert np.isinf(got[5])


@pytest.mark.parametrize("name,expected", [("rank7", 1.2), ("rank48", 1.2)])
def test_oracle_error_gate_config1(name, expected):
    """Config 1 (512x1024x1024, A~N(0,1), W~N(0,0.02)): the reduced-rank
    error stays within 1.2x of a BF16 product's error against FP64."""
    A, W, _ = make_linear_inputs(512, 1024, 1024, seed=0)
    a, w = f32(A).astype(np.float64), f32(W).astype(np.float64)
    exact = a @ w.T
    candidate = oracle.linear(name, f32(A), f32(W))
    native = oracle.bf16_round((a @ w.T).astype(np.float32))
    ratio = oracle.relative_l2(candidate, exact) / oracle.relative_l2(native, exact)
    assert np.isfinite(candidate).all()
    assert ratio < expected
