"""Pin the CPU oracle's FP16 plain-mm path to the reference's own kernels.

``tests/golden/make_golden_mm.py`` ran the reference's generated Triton
kernels with FP16 operands as its ``Rank7Plan.run`` / ``Rank49Plan.run`` do:
the left transform of ``A[M, K]``, the right transform of the contiguous
``B[K, N]`` and the output transform into FP16, plus the FP16 linear's
weight transform of ``weight[N, K]`` and its biased output transform.  The
oracle must reproduce every plane and every output bit for bit.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from inputs import digest, randn_fp16, random_products
from oracle import fmm_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
RECORD = json.loads((GOLDEN / "golden_mm.json").read_text())
SMALL = np.load(GOLDEN / "golden_mm.npz")


def _case_id(case):
    return f"{case['scheme']}-{'x'.join(map(str, case['shape']))}"


@pytest.mark.parametrize("case", RECORD["cases"], ids=_case_id)
def test_oracle_fp16_mm_matches_reference_kernels(case):
    name = case["scheme"]
    M, K, N = case["shape"]
    A = randn_fp16((M, K), case["seeds"]["A"])
    B = randn_fp16((K, N), case["seeds"]["B"])
    assert digest(A) == case["inputs"]["A"], "input generation drifted"
    assert digest(B) == case["inputs"]["B"]
    L = oracle.left_transform(name, A.float().numpy())
    R = oracle.right_transform(name, B.float().numpy())
    assert digest(L.view(np.int16)) == case["left"]
    assert digest(R.view(np.int16)) == case["right"]
    s, rank = oracle.scheme_circuits(name)[:2]
    bm, _, bn = oracle.block_dims(M, K, N, s)
    P = random_products(rank, bm, bn, seed=case["seeds"]["P"])
    assert digest(P) == case["inputs"]["P"]
    C = oracle.output_transform(name, P.numpy(), M, N, out_dtype="fp16").astype(np.float16)
    assert digest(C.view(np.int16)) == case["output"]
    # FP16 linear: native weight[N, K] = B^T and an FP16 bias
    Rw = oracle.weight_transform(name, B.t().contiguous().float().numpy())
    assert digest(Rw.view(np.int16)) == case["weight"]
    bias = randn_fp16((N,), case["seeds"]["bias"], 0.02)
    assert digest(bias) == case["inputs"]["bias"]
    Cb = oracle.output_transform(name, P.numpy(), M, N, bias.float().numpy(), out_dtype="fp16")
    assert digest(Cb.astype(np.float16).view(np.int16)) == case["output_bias"]
    key = f"{name}_{M}x{K}x{N}"
    if key + "_left" in SMALL:
        np.testing.assert_array_equal(L.view(np.int16), SMALL[key + "_left"])
        np.testing.assert_array_equal(R.view(np.int16), SMALL[key + "_right"])
        np.testing.assert_array_equal(C.view(np.int16), SMALL[key + "_output"])
        np.testing.assert_array_equal(Cb.astype(np.float16).view(np.int16), SMALL[key + "_output_bias"])


def test_fixtures_cover_the_fp16_plan_schemes():
    assert {c["scheme"] for c in RECORD["cases"]} == {"rank7", "rank49"}
    assert len(RECORD["cases"]) == 6
