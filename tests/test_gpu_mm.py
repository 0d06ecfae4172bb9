"""Plain-mm API and FP16 plans on the GPU (mirrors the reference's
tests/test_rdna3.py:406-484 and the FP16 side of its plans)."""

import numpy as np
import pytest
import torch

from inputs import f32, make_linear_inputs, random_products
from oracle import fmm_oracle as oracle
from rdna3_fastmm import _native, external_mm
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)
PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy()


def _rel(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b))


@pytest.mark.parametrize("name", list(PLANS))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(5, 6, 7), (257, 263, 269), (64, 200, 96)], ids=lambda s: "x".join(map(str, s)))
def test_right_kn_transform_matches_oracle_bitwise(name, dtype, shape):
    """fmm_transform_b(B) makes the planes of fmm_transform_w(B^T), bit for bit."""
    M, K, N = shape
    _, W, _ = make_linear_inputs(M, K, N, seed=4)
    B = W.t().contiguous().to(dtype)  # [K, N]
    s = MatrixShape.from_dimensions(M, K, N, PLANS[name].scheme_size)
    Rt = torch.full((PLANS[name].rank, s.block_columns, s.inner_pitch), float("nan"), device=DEVICE,
                    dtype=torch.float16)
    _native.transform_b(name, B.to(DEVICE), Rt)
    torch.cuda.synchronize()
    ref = oracle.weight_transform(name, B.t().float().numpy())  # [R, bk, bn]
    bk = s.block_inner
    np.testing.assert_array_equal(_bits(Rt[:, :, :bk].transpose(1, 2)), ref.view(np.int16))
    assert torch.all(Rt[:, :, bk:] == 0)


@pytest.mark.parametrize("variant", ["staged", "register"])
@pytest.mark.parametrize("name", ["rank7", "rank49"])
def test_fp16_left_transform_and_fp16_reconstruct_match_oracle(name, variant, monkeypatch):
    monkeypatch.setenv("FMM_RECONSTRUCT_VARIANT", variant)  # rank 49: TMA-staged or register kernel
    M, K, N = 257, 263, 269
    A, _, bias = make_linear_inputs(M, K, N, seed=6, bias=True)
    A, bias = A.to(torch.float16), bias.to(torch.float16)
    plan_type = PLANS[name]
    s = MatrixShape.from_dimensions(M, K, N, plan_type.scheme_size)
    L = torch.empty((plan_type.rank, s.block_rows, s.inner_pitch), device=DEVICE, dtype=torch.float16)
    _native.transform_a(name, A.to(DEVICE), L)
    products = random_products(plan_type.rank, s.block_rows, s.block_columns, seed=8)
    P = torch.zeros((plan_type.rank, s.block_rows, s.column_pitch), device=DEVICE, dtype=torch.float16)
    P[:, :, : s.block_columns] = products.to(DEVICE)
    C = torch.empty((M, N), device=DEVICE, dtype=torch.float16)
    _native.reconstruct(name, P, M, N, bias.to(DEVICE), C)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(L[:, :, : s.block_inner]),
                                  oracle.left_transform(name, A.float().numpy()).view(np.int16))
    ref = oracle.output_transform(name, products.numpy(), M, N, bias.float().numpy(), out_dtype="fp16")
    np.testing.assert_array_equal(_bits(C), ref.astype(np.float16).view(np.int16))


@pytest.mark.parametrize("plan_type", [Rank7Plan, Rank49Plan])
def test_fp16_run_and_run_packed_match_exact_small_product(plan_type):
    torch.manual_seed(11)
    left = torch.randint(-2, 3, (5, 6), device=DEVICE).to(torch.float16)
    right = torch.randint(-2, 3, (6, 7), device=DEVICE).to(torch.float16)
    expected = (left.float() @ right.float()).half()
    plan = plan_type(5, 6, 7, DEVICE)
    ws = plan.allocate_workspace(max_free_memory_fraction=0.1)
    packed = plan.pack_right(right, max_free_memory_fraction=0.1)
    pws = plan.allocate_workspace(max_free_memory_fraction=0.1, prepacked_right=True)
    for _ in range(3):
        assert torch.equal(plan.run(left, right, ws), expected)
        assert torch.equal(plan.run_packed(left, packed, pws), expected)
    snapshot = plan.run_packed(left, packed, pws).clone()
    right.zero_()
    assert torch.equal(plan.run_packed(left, packed, pws), snapshot)
    s = plan.shape
    assert plan.packed_right_bytes == plan.rank * s.block_columns * s.inner_pitch * 2
    assert packed.source_shape == (6, 7)


@pytest.mark.parametrize("plan_type", [Rank7Plan, Rank49Plan])
def test_fp16_random_nondivisible_shape_has_bounded_error(plan_type):
    torch.manual_seed(7)
    left = torch.randn((257, 263), device=DEVICE, dtype=torch.float16)
    right = torch.randn((263, 269), device=DEVICE, dtype=torch.float16)
    reference = left.double() @ right.double()
    plan = plan_type(257, 263, 269, DEVICE)
    dynamic = plan.run(left, right, plan.allocate_workspace(0.1))
    packed = plan.run_packed(left, plan.pack_right(right, 0.1), plan.allocate_workspace(0.1, prepacked_right=True))
    assert torch.isfinite(dynamic).all()
    assert _rel(dynamic, reference) < 5e-3
    assert torch.equal(dynamic, packed)


def test_fp16_linear_plan_with_bias():
    x, w, b = (t.to(torch.float16).to(DEVICE) for t in make_linear_inputs(257, 263, 269, seed=19, bias=True))
    reference = x.double() @ w.double().T + b.double()
    plan = Rank7Plan(257, 263, 269, DEVICE)
    out = plan.run_linear(x, w, plan.allocate_workspace(0.1), b)
    assert out.dtype == torch.float16
    assert _rel(out, reference) < 5e-3


def test_rank48_refuses_fp16_plans():
    with pytest.raises(ValueError, match="does not support"):
        Rank48Plan(8, 8, 8, DEVICE)


def test_external_matmul_runs_the_plan_for_an_admitted_shape(monkeypatch):
    monkeypatch.setattr(Rank49Plan, "dynamic_shapes", frozenset({(64, 80, 96)}))
    left = torch.randn((64, 80), device=DEVICE, dtype=torch.float16)
    right = torch.randn((80, 96), device=DEVICE, dtype=torch.float16)
    out = torch.empty((64, 96), device=DEVICE, dtype=torch.float16)
    with torch.no_grad():
        assert external_mm.is_rank49_dynamic_eligible(left, right, out)
        external_mm.rdna3_rank49_dynamic_v1_out(left, right, out=out)
    assert _rel(out, left.double() @ right.double()) < 5e-3
