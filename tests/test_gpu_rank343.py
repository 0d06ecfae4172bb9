"""Rank-343 <8,8,8> FP16 square path on B200 vs the CPU oracle (through the
C ABI and the plan API), mirroring the reference's rank-343 GPU tests
(``tests/test_rdna3.py:713-752``).

* left / right / weight transforms: bit for bit (the oracle is pinned to the
  reference's ``rank343_8x8x8.py`` kernels by ``test_oracle_rank343.py``);
* reconstruct: a tensor-core product with the +-1 coefficient matrix (as the
  reference's MFMA reconstruction), FP32 accumulation in the hardware's
  order: within one FP16 ulp of the oracle's ascending-order sum, nearly
  all elements equal;
* whole products: within the leaf-GEMM tolerance of the oracle and within
  5e-3 relative L2 of an FP64 product; dynamic == packed bitwise.
"""

import numpy as np
import pytest
import torch

from inputs import random_products, randn_fp16
from oracle import fmm_oracle as oracle
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank343Plan

pytestmark = pytest.mark.gpu

SHAPES = [(5, 6, 7), (17, 19, 23), (67, 71, 73), (257, 263, 269), (512, 520, 536)]


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy()


def _planes(M, K, N):
    s = MatrixShape.from_dimensions(M, K, N, 8)
    nan = float("nan")
    L = torch.full((343, s.block_rows, s.inner_pitch), nan, device="cuda", dtype=torch.float16)
    Rt = torch.full((343, s.block_columns, s.inner_pitch), nan, device="cuda", dtype=torch.float16)
    P = torch.full((343, s.block_rows, s.column_pitch), nan, device="cuda", dtype=torch.float16)
    return s, L, Rt, P


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_rank343_transforms_match_oracle_bitwise(shape):
    M, K, N = shape
    A = randn_fp16((M, K), 0)
    B = randn_fp16((K, N), 1)
    s, L, Rt, _ = _planes(M, K, N)
    bk = s.block_inner
    _native.transform_a("rank343", A.cuda(), L)
    _native.transform_b("rank343", B.cuda(), Rt)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(L[:, :, :bk]),
                                  oracle.left_transform("rank343", A.float().numpy()).view(np.int16))
    ref_R = oracle.right_transform("rank343", B.float().numpy())
    np.testing.assert_array_equal(_bits(Rt[:, :, :bk].transpose(1, 2)), ref_R.view(np.int16))
    assert torch.all(L[:, :, bk:] == 0) and torch.all(Rt[:, :, bk:] == 0)
    # weight layout (native [N, K]) gives the same planes
    Rw = torch.full_like(Rt, float("nan"))
    _native.transform_w("rank343", B.t().contiguous().cuda(), Rw)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(Rw), _bits(Rt))


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_rank343_reconstruct_matches_oracle_bitwise(shape):
    M, K, N = shape
    s, _, _, P = _planes(M, K, N)
    bm, bn = s.block_rows, s.block_columns
    prod = random_products(343, bm, bn, seed=3)
    P[:, :, :bn] = prod.cuda()
    P[:, :, bn:] = 0
    C = torch.empty((M, N), device="cuda", dtype=torch.float16)
    _native.reconstruct("rank343", P, M, N, None, C)
    torch.cuda.synchronize()
    ref = oracle.output_transform("rank343", prod.numpy(), M, N, None, "fp16").astype(np.float16)
    got = C.cpu().numpy()
    ulp = np.spacing(np.abs(ref)).astype(np.float64)
    assert np.all(np.abs(got.astype(np.float64) - ref.astype(np.float64)) <= ulp)
    assert np.mean(got == ref) > 0.99


@pytest.mark.parametrize("shape", [(257, 263, 269), (1030, 64, 2050)], ids=lambda s: "x".join(map(str, s)))
def test_rank343_reconstruct_with_bias(shape):
    M, K, N = shape
    s, _, _, P = _planes(M, K, N)
    bm, bn = s.block_rows, s.block_columns
    prod = random_products(343, bm, bn, seed=7)
    P[:, :, :bn] = prod.cuda()
    P[:, :, bn:] = 0
    bias = randn_fp16((N,), 9)
    C = torch.empty((M, N), device="cuda", dtype=torch.float16)
    _native.reconstruct("rank343", P, M, N, bias.cuda(), C)
    torch.cuda.synchronize()
    ref = oracle.output_transform("rank343", prod.numpy(), M, N, bias.float().numpy(), "fp16")
    ref = ref.astype(np.float16)
    got = C.cpu().numpy()
    ulp = np.spacing(np.abs(ref)).astype(np.float64)
    assert np.all(np.abs(got.astype(np.float64) - ref.astype(np.float64)) <= ulp)


def _gemm_tolerance(L, R):
    a = np.abs(L.astype(np.float64))
    b = np.abs(R.astype(np.float64))
    return np.matmul(a, b)


@pytest.mark.parametrize("shape", [(67, 71, 73), (257, 263, 269), (1024, 1032, 1040)],
                         ids=lambda s: "x".join(map(str, s)))
def test_rank343_plan_matches_oracle(shape):
    M, K, N = shape
    A = randn_fp16((M, K), 0)
    B = randn_fp16((K, N), 1)
    plan = Rank343Plan(M, K, N, torch.device("cuda"))
    Ad, Bd = A.cuda(), B.cuda()
    dynamic = plan.run(Ad, Bd, plan.allocate_workspace(0.5))
    packed = plan.run_packed(Ad, plan.pack_right(Bd, 0.5), plan.allocate_workspace(0.5, prepacked_right=True))
    torch.cuda.synchronize()
    assert torch.equal(dynamic.view(torch.int16), packed.view(torch.int16))
    ref = oracle.matmul("rank343", A.float().numpy(), B.float().numpy())
    exact = A.double().numpy() @ B.double().numpy()
    got = dynamic.float().cpu().numpy()
    assert oracle.relative_l2(got, ref) < 2e-3
    assert oracle.relative_l2(got, exact) < 5e-3
    assert np.isfinite(got).all()


def test_rank343_dynamic_and_packed_match_exact_small_product():
    torch.manual_seed(17)
    left = torch.randint(-2, 3, (5, 6), device="cuda").to(torch.float16)
    right = torch.randint(-2, 3, (6, 7), device="cuda").to(torch.float16)
    reference = (left.float() @ right.float()).half()
    plan = Rank343Plan(5, 6, 7, torch.device("cuda"))
    torch.testing.assert_close(plan.run(left, right, plan.allocate_workspace(0.1)), reference,
                               rtol=0, atol=0.001)
    packed = plan.pack_right(right, 0.1)
    torch.testing.assert_close(plan.run_packed(left, packed, plan.allocate_workspace(0.1, prepacked_right=True)),
                               reference, rtol=0, atol=0.001)


def test_rank343_rejects_bfloat16_inputs():
    with pytest.raises(ValueError, match="does not support"):
        Rank343Plan(8, 8, 8, torch.device("cuda"), dtype=torch.bfloat16, compute_dtype=torch.float16)
    A = torch.zeros((16, 16), device="cuda", dtype=torch.bfloat16)
    L = torch.empty((343, 2, 8), device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="FP16"):
        _native.transform_a("rank343", A, L)


def test_rank343_reconstruct_rejects_unaligned_products():
    """The staged kernel copies 16-byte chunks: P must be 16-byte aligned."""
    M, K, N = 67, 71, 73
    s = MatrixShape.from_dimensions(M, K, N, 8)
    flat = torch.zeros(343 * s.block_rows * s.column_pitch + 1, device="cuda", dtype=torch.float16)
    shifted = flat[1:].view(343, s.block_rows, s.column_pitch)  # 2-byte offset
    C = torch.empty((M, N), device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="16-byte aligned"):
        _native.reconstruct("rank343", shifted, M, N, None, C)
