"""Edge shapes through the whole CUDA path, against the CPU oracle:
single rows/columns, K smaller than one 64-wide k-block, dimensions below
the scheme size (blocks that are all padding), and very skinny products."""

import numpy as np
import pytest
import torch

from inputs import f32, make_linear_inputs
from oracle import fmm_oracle as oracle
from rdna3_fastmm.runtime import Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu
PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
SHAPES = [(1, 1, 1), (1, 7, 3), (3, 1, 5), (2, 2, 2), (4, 3, 4), (1, 4096, 8), (300, 5, 2), (9, 130, 1)]


@pytest.mark.parametrize("name", list(PLANS))
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_edge_shapes_match_oracle(name, shape):
    M, K, N = shape
    A, W, bias = make_linear_inputs(M, K, N, seed=2, bias=True)
    plan = PLANS[name](M, K, N, torch.device("cuda"), dtype=torch.bfloat16, compute_dtype=torch.float16)
    dyn = plan.run_linear(A.cuda(), W.cuda(), plan.allocate_workspace(0.1), bias.cuda())
    packed = plan.run_linear_packed(A.cuda(), plan.pack_weight(W.cuda(), 0.1),
                                    plan.allocate_workspace(0.1, prepacked_right=True), bias.cuda())
    torch.cuda.synchronize()
    ref = oracle.linear(name, f32(A), f32(W), f32(bias))
    got = dyn.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert torch.equal(dyn, packed)
    # tiny products are dominated by single roundings: compare elementwise
    np.testing.assert_allclose(got, ref, rtol=2e-2, atol=2e-2)


def test_leading_dims_and_noncontiguous_input_through_the_op():
    from rdna3_fastmm.linear import rdna3_rank7_linear

    x = torch.randn((3, 40, 64), device="cuda", dtype=torch.bfloat16).transpose(0, 1)  # non-contiguous
    w = torch.randn((48, 64), device="cuda", dtype=torch.bfloat16) * 0.1
    out = rdna3_rank7_linear(x, w)
    ref = x.double() @ w.double().T
    assert out.shape == (40, 3, 48)
    rel = torch.linalg.vector_norm(out.double() - ref) / torch.linalg.vector_norm(ref)
    assert rel < 5e-3
