"""The rank-49 ``(bfloat16, bfloat16)`` precision pair on B200, through the C ABI.

The reference's ``Rank49Plan`` accepts BF16 inputs with BF16 transform planes
and BF16 leaf products (``src/rdna3_fastmm/runtime.py:852-858``); with
``dtype=torch.bfloat16`` and no ``compute_dtype`` that is the pair a plan
resolves to.  Here:

* the transforms (left, native weight, contiguous right) and the reconstruct
  (both kernels, with and without bias) must equal the oracle's BF16-plane
  mode bit for bit -- the oracle mode is pinned to the reference's kernels by
  ``test_oracle_golden_bf16.py``;
* the BF16 leaf GEMM (tcgen05 with BF16 operands) is held to one BF16 ulp of
  rounding plus the worst-case FP32 accumulation bound of an FP64 product;
* whole linears stay within 2e-3 relative L2 of the oracle's BF16-plane linear
  (products may differ by an ulp; BF16 has 8 significand bits, so the
  path's own error against FP64 is ~1.6e-2, well above the FP16-leaf pair's);
* dynamic and prepacked outputs are bitwise identical.
"""

import numpy as np
import pytest
import torch

from inputs import f32, make_linear_inputs
from oracle import fmm_oracle as oracle
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu

SHAPES = [(5, 6, 7), (17, 19, 23), (257, 263, 269), (64, 128, 256), (130, 1030, 514)]


def _planes(M, K, N):
    s = MatrixShape.from_dimensions(M, K, N, 4)
    nan = float("nan")
    L = torch.full((49, s.block_rows, s.inner_pitch), nan, device="cuda", dtype=torch.bfloat16)
    Rt = torch.full((49, s.block_columns, s.inner_pitch), nan, device="cuda", dtype=torch.bfloat16)
    P = torch.full((49, s.block_rows, s.column_pitch), nan, device="cuda", dtype=torch.bfloat16)
    return s, L, Rt, P


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy()


def _oracle_bits(x):
    return oracle.bf16_bits(x).view(np.int16)


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_bf16_transforms_match_oracle_bitwise(shape):
    M, K, N = shape
    A, W, _ = make_linear_inputs(M, K, N, seed=0)
    s, L, Rt, _ = _planes(M, K, N)
    _native.transform_a("rank49", A.cuda(), L)
    _native.transform_w("rank49", W.cuda(), Rt)
    _, L2, R2, _ = _planes(M, K, N)
    _native.transform_aw("rank49", A.cuda(), L2, W.cuda(), R2)
    _, _, Rkn, _ = _planes(M, K, N)
    _native.transform_b("rank49", W.t().contiguous().cuda(), Rkn)
    torch.cuda.synchronize()
    bk = s.block_inner
    ref_L = oracle.left_transform("rank49", f32(A), planes="bf16")
    ref_R = oracle.weight_transform("rank49", f32(W), planes="bf16")  # [R, bk, bn]
    np.testing.assert_array_equal(_bits(L[:, :, :bk]), _oracle_bits(ref_L))
    np.testing.assert_array_equal(_bits(Rt[:, :, :bk].transpose(1, 2)), _oracle_bits(ref_R))
    assert torch.equal(L.view(torch.int16), L2.view(torch.int16))
    assert torch.equal(Rt.view(torch.int16), R2.view(torch.int16))
    assert torch.equal(Rt.view(torch.int16), Rkn.view(torch.int16))
    assert torch.all(L[:, :, bk:] == 0) and torch.all(Rt[:, :, bk:] == 0)


@pytest.mark.parametrize("variant", ["staged", "register"])
@pytest.mark.parametrize("shape", SHAPES + [(2052, 64, 4100), (1029, 64, 2064)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("with_bias", [False, True])
def test_bf16_reconstruct_matches_oracle_bitwise(shape, with_bias, variant, monkeypatch):
    monkeypatch.setenv("FMM_RECONSTRUCT_VARIANT", variant)
    M, K, N = shape
    _, _, bias = make_linear_inputs(M, K, N, seed=0, bias=True)
    s, _, _, P = _planes(M, K, N)
    g = torch.Generator().manual_seed(3)
    products = torch.randn((49, s.block_rows, s.block_columns), generator=g).to(torch.bfloat16)
    P.zero_()
    P[:, :, : s.block_columns] = products.cuda()
    C = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    _native.reconstruct("rank49", P, M, N, bias.cuda() if with_bias else None, C)
    torch.cuda.synchronize()
    ref = oracle.output_transform("rank49", products.float().numpy(), M, N,
                                  f32(bias) if with_bias else None)
    np.testing.assert_array_equal(_bits(C), _oracle_bits(ref))


@pytest.mark.parametrize("variant", ["single", "pair256", "pair256k128", "pair256-tma", "pair256k128-tma",
                                     "pair192k128-tma", "pair128k128-tma"])
@pytest.mark.parametrize(
    "rank,bm,bn,bk",
    [(1, 128, 256, 64), (7, 65, 68, 66), (3, 300, 600, 200), (49, 64, 72, 130), (5, 700, 900, 520)],
)
def test_bf16_leaf_gemm_matches_fp64_products(rank, bm, bn, bk, variant, monkeypatch):
    variant, _, epilogue = variant.partition("-")
    monkeypatch.setenv("FMM_LEAF_GEMM_VARIANT", variant)
    monkeypatch.setenv("FMM_LEAF_GEMM_EPILOGUE", epilogue or "rows")
    g = torch.Generator().manual_seed(rank * 1000 + bm)
    ldk = -(-bk // 8) * 8
    ldp = -(-bn // 8) * 8
    L = torch.zeros((rank, bm, ldk), dtype=torch.bfloat16)
    Rt = torch.zeros((rank, bn, ldk), dtype=torch.bfloat16)
    L[:, :, :bk] = torch.randn((rank, bm, bk), generator=g).to(torch.bfloat16)
    Rt[:, :, :bk] = torch.randn((rank, bn, bk), generator=g).to(torch.bfloat16)
    if ldk > bk:  # the GEMM must not read the pitch padding
        L[:, :, bk:] = float("nan")
        Rt[:, :, bk:] = float("nan")
    P = torch.full((rank, bm, ldp), float("nan"), device="cuda", dtype=torch.bfloat16)
    _native.leaf_gemm(rank, L.cuda(), Rt.cuda(), bm, bn, bk, P)
    torch.cuda.synchronize()
    a, b = L[:, :, :bk].double(), Rt[:, :, :bk].double().transpose(1, 2)
    exact = torch.matmul(a, b)
    magnitude = torch.matmul(a.abs(), b.abs())
    got = P[:, :, :bn].cpu().double()
    assert torch.isfinite(got).all()
    # BF16 rounding of the product (half an ulp of 8 significand bits,
    # doubled for slack) plus the worst-case FP32 accumulation over bk terms
    ulp = torch.clamp(exact.abs(), min=2.0**-126) * 2.0**-7
    bound = ulp + (bk + 2) * 2.0**-23 * magnitude
    assert torch.all((got - exact).abs() <= bound)


@pytest.mark.parametrize("shape", [(5, 6, 7), (257, 263, 269), (512, 1024, 1024)],
                         ids=lambda s: "x".join(map(str, s)))
def test_bf16_linear_matches_oracle_and_prepacked(shape):
    M, K, N = shape
    A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=True)
    dev = torch.device("cuda")
    plan = Rank49Plan(M, K, N, dev, dtype=torch.bfloat16)  # resolves to (bf16, bf16)
    assert plan.compute_dtype == torch.bfloat16
    ws = plan.allocate_workspace(0.5)
    assert ws.left_transformed.dtype == torch.bfloat16
    out = plan.run_linear(A.cuda(), W.cuda(), ws, bias.cuda())
    packed = plan.pack_weight(W.cuda(), 0.5)
    out_packed = plan.run_linear_packed(A.cuda(), packed, plan.allocate_workspace(0.5, prepacked_right=True),
                                        bias.cuda())
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out_packed.view(torch.int16))
    ref = oracle.linear("rank49", f32(A), f32(W), f32(bias), planes="bf16")
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.relative_l2(got, ref) < 2e-3
    exact = f32(A).astype(np.float64) @ f32(W).astype(np.float64).T + f32(bias)
    assert oracle.relative_l2(got, exact) < 5e-2


def test_bf16_plain_mm_matches_linear():
    """The mm API (contiguous right matrix) with BF16 planes gives the linear's bits."""
    M, K, N = 130, 1030, 514
    A, W, _ = make_linear_inputs(M, K, N, seed=1)
    plan = Rank49Plan(M, K, N, torch.device("cuda"), dtype=torch.bfloat16, compute_dtype=torch.bfloat16)
    ws = plan.allocate_workspace(0.5)
    out_mm = plan.run(A.cuda(), W.t().contiguous().cuda(), ws)
    out_lin = plan.run_linear(A.cuda(), W.cuda(), plan.allocate_workspace(0.5))
    packed = plan.pack_right(W.t().contiguous().cuda(), 0.5)
    out_packed = plan.run_packed(A.cuda(), packed, plan.allocate_workspace(0.5, prepacked_right=True))
    torch.cuda.synchronize()
    assert torch.equal(out_mm.view(torch.int16), out_lin.view(torch.int16))
    assert torch.equal(out_mm.view(torch.int16), out_packed.view(torch.int16))


def test_bf16_planes_are_rank49_only():
    """Only Rank49Plan offers BF16 planes (as in the reference); the C ABI
    refuses them for the other circuit schemes."""
    dev = torch.device("cuda")
    for plan_type in (Rank7Plan, Rank48Plan):
        with pytest.raises(ValueError):
            plan_type(8, 8, 8, dev, dtype=torch.bfloat16, compute_dtype=torch.bfloat16)
    A = torch.zeros((8, 8), device="cuda", dtype=torch.bfloat16)
    L = torch.zeros((7, 4, 8), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="rank 49 only"):
        _native.transform_a("rank7", A, L)
