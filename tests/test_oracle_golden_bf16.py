"""Pin the oracle's BF16-plane mode to the reference's own kernels.

The reference's ``Rank49Plan`` runs its rank-49 transforms with BF16 planes
for the ``(bfloat16, bfloat16)`` precision pair.  ``golden/make_golden_bf16.py``
ran those generated Triton kernels (FP32 stores rounded to BF16 by torch,
which is what a GPU's BF16 store does); the oracle with ``planes="bf16"`` must
reproduce every left and weight plane and every output, with and without
bias, bit for bit.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from inputs import digest, f32, make_linear_inputs
from oracle import fmm_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
RECORD = json.loads((GOLDEN / "golden_bf16.json").read_text())
SMALL = np.load(GOLDEN / "golden_bf16.npz")


def _bits(x: np.ndarray) -> np.ndarray:
    """float32 arrays holding BF16 values -> their int16 bit patterns."""
    return oracle.bf16_bits(x).view(np.int16)


def _products(rank: int, bm: int, bn: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn((rank, bm, bn), generator=g, dtype=torch.float32).to(torch.bfloat16)


@pytest.mark.parametrize("case", RECORD["cases"], ids=lambda c: "x".join(map(str, c["shape"])))
def test_bf16_planes_match_reference_kernels(case):
    M, K, N = case["shape"]
    A, W, bias = make_linear_inputs(M, K, N, seed=case["seed"], bias=True)
    assert digest(A) == case["inputs"]["A"], "input generation drifted"
    assert digest(W) == case["inputs"]["W"]
    L = oracle.left_transform("rank49", f32(A), planes="bf16")
    R = oracle.weight_transform("rank49", f32(W), planes="bf16")
    assert digest(_bits(L)) == case["left"]
    assert digest(_bits(R)) == case["weight"]
    bm, _, bn = oracle.block_dims(M, K, N, 4)
    P = _products(49, bm, bn, case["product_seed"])
    assert digest(P) == case["inputs"]["P"]
    P32 = P.float().numpy()
    C = oracle.output_transform("rank49", P32, M, N)
    Cb = oracle.output_transform("rank49", P32, M, N, f32(bias))
    assert digest(_bits(C)) == case["output"]
    assert digest(_bits(Cb)) == case["output_bias"]
    key = f"rank49_{M}x{K}x{N}"
    if key + "_left" in SMALL:
        np.testing.assert_array_equal(_bits(L), SMALL[key + "_left"])
        np.testing.assert_array_equal(_bits(R), SMALL[key + "_weight"])
        np.testing.assert_array_equal(_bits(Cb), SMALL[key + "_output_bias"])


def test_bf16_planes_differ_from_fp16_planes():
    """The BF16 mode really rounds to BF16: planes differ from the FP16 ones
    and every value is BF16-representable."""
    A, W, _ = make_linear_inputs(17, 19, 23, seed=0)
    L16 = oracle.left_transform("rank49", f32(A))
    Lbf = oracle.left_transform("rank49", f32(A), planes="bf16")
    assert not np.array_equal(L16.astype(np.float32), Lbf)
    np.testing.assert_array_equal(oracle.bf16_round(Lbf), Lbf)
