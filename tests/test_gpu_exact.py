"""Known-answer tests on B200 over many shapes: every scheme is an exact
identity over the integers, so for small-integer inputs the whole path --
transforms, tcgen05 leaf GEMM (FP32 accumulation of integers is exact),
recombination -- must return the exact product bit for bit, for ragged shapes
of every size class (the reference's exact 5x6x7 test, tests/test_rdna3.py:406-430,
generalised)."""

import numpy as np
import pytest
import torch

from rdna3_fastmm.runtime import Rank7Plan, Rank48Plan, Rank49Plan, Rank343Plan

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)
PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}


def _shapes(seed, count, k_max=300):
    rng = np.random.default_rng(seed)
    return [(int(rng.integers(1, 300)), int(rng.integers(1, k_max)), int(rng.integers(1, 300)))
            for _ in range(count)]


@pytest.mark.parametrize("name", list(PLANS))
@pytest.mark.parametrize("shape", _shapes(2024, 8), ids=lambda s: "x".join(map(str, s)))
def test_linear_of_small_integers_is_exact(name, shape):
    M, K, N = shape
    g = torch.Generator().manual_seed(M * 7919 + K * 31 + N)
    # BF16 holds integers exactly up to 256: at most 250 nonzero terms plus a bias of at most 3.
    # Every FP16 plane value stays below 2048 (FP16's exact integers) for these magnitudes.
    A = torch.randint(-1, 2, (M, K), generator=g).to(torch.bfloat16)
    W = torch.randint(-1, 2, (N, K), generator=g).to(torch.bfloat16)
    if K > 250:
        A[:, 250:] = 0
    bias = torch.randint(-3, 4, (N,), generator=g).to(torch.bfloat16)
    expected = (A.double() @ W.double().T + bias.double()).to(torch.bfloat16)
    plan = PLANS[name](M, K, N, DEVICE, dtype=torch.bfloat16, compute_dtype=torch.float16)
    got = plan.run_linear(A.to(DEVICE), W.to(DEVICE), plan.allocate_workspace(0.5), bias.to(DEVICE))
    packed = plan.pack_weight(W.to(DEVICE), 0.5)
    got_packed = plan.run_linear_packed(A.to(DEVICE), packed, plan.allocate_workspace(0.5, prepacked_right=True),
                                        bias.to(DEVICE))
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), expected)
    assert torch.equal(got_packed.cpu(), expected)


# K <= 200: products of rank-343 planes stay below 2048, FP16's exact integers
@pytest.mark.parametrize("shape", _shapes(343, 6, k_max=200), ids=lambda s: "x".join(map(str, s)))
def test_rank343_mm_of_small_integers_is_exact(shape):
    M, K, N = shape
    g = torch.Generator().manual_seed(M + 1000 * K + 7 * N)
    A = torch.randint(-1, 2, (M, K), generator=g).to(torch.float16)
    B = torch.randint(-1, 2, (K, N), generator=g).to(torch.float16)
    expected = (A.double() @ B.double()).to(torch.float16)
    plan = Rank343Plan(M, K, N, DEVICE)
    got = plan.run(A.to(DEVICE), B.to(DEVICE), plan.allocate_workspace(0.5))
    packed = plan.pack_right(B.to(DEVICE), 0.5)
    got_packed = plan.run_packed(A.to(DEVICE), packed, plan.allocate_workspace(0.5, prepacked_right=True))
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), expected)
    assert torch.equal(got_packed.cpu(), expected)
