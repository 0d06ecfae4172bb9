"""Parity at the benchmark configurations' full sizes.

The CPU oracle cannot run a whole 8192^3 linear in seconds, but every stage
of the path is position-wise, so sampled positions pin the full-size launch:

* row block ``i`` of the left planes depends only on rows ``p_r * bm + i`` of
  ``A`` (one per block row ``p_r``): the oracle's left transform of that
  ``s``-row matrix must give ``L[:, i, :]`` bit for bit;
* likewise column block ``j`` of the weight planes and rows
  ``p_c * bn + j`` of ``W``;
* row ``i`` of the products and the output rows ``p_r * bm + i`` for the
  output transform (bit for bit, with the bias);
* the leaf GEMM's sampled rows against an FP64 product of the same planes
  within one ulp of the plane format plus the FP32 accumulation bound;
* the whole call through the plan API, dynamic and prepacked, equals the
  staged launches bit for bit.

Every configuration runs with FP16 planes; c4 (rank 49) also runs with the
BF16 planes of the reference's ``(bfloat16, bfloat16)`` precision pair.
Sampled block rows always include the first and the last (padded) one.  The
rank-343 FP16 square product is checked the same way at 16384^3, its
tensor-core reconstruct within one FP16 ulp plus the FP32 accumulation bound
of the 343-term sum.
"""

import numpy as np
import pytest
import torch

from inputs import f32, make_linear_inputs, randn_fp16
from oracle import fmm_oracle as oracle
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan, Rank343Plan

pytestmark = pytest.mark.gpu

PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
# (scheme, M, K, N, bias): the benchmark configurations c2, c3, c4, c5a, c5b
CONFIGS = {
    "c2": ("rank7", 4096, 4096, 12288, False),
    "c3": ("rank7", 4992, 16384, 4096, True),
    "c4": ("rank49", 8214, 12288, 4608, False),
    "c5a": ("rank48", 8192, 8192, 8192, False),
    "c5b": ("rank48", 65536, 4608, 12288, False),
}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy()


def _sample(n: int, count: int, seed: int) -> list[int]:
    rng = np.random.default_rng(seed)
    picked = set(rng.choice(n, size=min(count, n), replace=False).tolist()) | {0, n - 1}
    return sorted(picked)


def _block_rows(X: torch.Tensor, s: int, pitch: int, index: int) -> torch.Tensor:
    """Rows ``p * pitch + index`` of X for p < s; missing rows (past the end)
    are zero, which is the zero padding of the last block."""
    out = torch.zeros((s, X.shape[1]), dtype=X.dtype)
    for p in range(s):
        row = p * pitch + index
        if row < X.shape[0]:
            out[p] = X[row]
    return out


# (config, planes): every configuration with FP16 planes, and c4 (rank 49)
# with the BF16 planes of the reference's (bfloat16, bfloat16) precision pair
CASES = [(config, "fp16") for config in CONFIGS] + [("c4", "bf16")]
PLANE_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _plane_bits(ref: np.ndarray, planes: str) -> np.ndarray:
    """Oracle planes (float16, or float32 holding BF16) -> int16 bit patterns."""
    return ref.view(np.int16) if planes == "fp16" else oracle.bf16_bits(ref).view(np.int16)


def _host_products(P: torch.Tensor) -> np.ndarray:
    """Device products -> the oracle's product input (float16, or float32
    holding the BF16 values)."""
    P = P.cpu()
    return P.numpy() if P.dtype == torch.float16 else P.float().numpy()


@pytest.mark.parametrize("config,planes", CASES, ids=lambda v: v)
def test_full_size_stages_match_oracle_on_sampled_positions(config, planes):
    name, M, K, N, with_bias = CONFIGS[config]
    plan_type = PLANS[name]
    pd = PLANE_DTYPES[planes]
    s_ = plan_type.scheme_size
    A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=with_bias)
    shape = MatrixShape.from_dimensions(M, K, N, s_)
    bm, bk, bn = shape.block_rows, shape.block_inner, shape.block_columns
    R = plan_type.rank
    dev = torch.device("cuda")
    Ad, Wd = A.to(dev), W.to(dev)
    bd = bias.to(dev) if with_bias else None
    L = torch.empty((R, bm, shape.inner_pitch), device=dev, dtype=pd)
    Rt = torch.empty((R, bn, shape.inner_pitch), device=dev, dtype=pd)
    P = torch.empty((R, bm, shape.column_pitch), device=dev, dtype=pd)
    C = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
    _native.transform_a(name, Ad, L)
    _native.transform_w(name, Wd, Rt)
    _native.leaf_gemm(R, L, Rt, bm, bn, bk, P)
    _native.reconstruct(name, P, M, N, bd, C)
    torch.cuda.synchronize()

    # left and weight transforms, bit for bit
    for i in _sample(bm, 6, seed=1):
        ref = oracle.left_transform(name, f32(_block_rows(A, s_, bm, i)), planes)  # [R, 1, bk]
        np.testing.assert_array_equal(_bits(L[:, i, :bk]), _plane_bits(ref[:, 0, :], planes))
    for j in _sample(bn, 6, seed=2):
        ref = oracle.weight_transform(name, f32(_block_rows(W, s_, bn, j)), planes)  # [R, bk, 1]
        np.testing.assert_array_equal(_bits(Rt[:, j, :bk]), _plane_bits(ref[:, :, 0], planes))

    # leaf products within the plane format's rounding + FP32 accumulation
    # bound (FP64 on the device: IEEE double products of the same planes)
    _leaf_rows_within_bound(L, Rt, P, _sample(bm, 4, seed=3), bk, bn)

    # output transform of the GPU's own products, bit for bit, bias included
    for i in _sample(bm, 6, seed=4):
        rows = [p * bm + i for p in range(s_) if p * bm + i < M]
        products = _host_products(P[:, i:i + 1, :bn])
        ref = oracle.output_transform(name, products, len(rows), N, f32(bias) if with_bias else None)
        np.testing.assert_array_equal(_bits(C[rows]), oracle.bf16_bits(ref).view(np.int16))
    assert torch.isfinite(C.float()).all()

    # the plan API (dynamic: paired input transforms; prepacked: packed weight)
    # gives the same bits as the staged launches
    plan = plan_type(M, K, N, dev, dtype=torch.bfloat16, compute_dtype=pd)
    del L, Rt, P
    ws = plan.allocate_workspace(max_free_memory_fraction=0.9)
    dynamic = plan.run_linear(Ad, Wd, ws, bd)
    assert torch.equal(dynamic.view(torch.int16), C.view(torch.int16))
    del ws, dynamic
    packed = plan.pack_weight(Wd, 0.9)
    ws = plan.allocate_workspace(max_free_memory_fraction=0.9, prepacked_right=True)
    prepacked = plan.run_linear_packed(Ad, packed, ws, bd)
    assert torch.equal(prepacked.view(torch.int16), C.view(torch.int16))


def _leaf_rows_within_bound(L, Rt, P, rows, bk, bn):
    """Sampled product rows against a device-FP64 product of the same planes:
    one ulp of the plane format (FP16: 11 significand bits; BF16: 8, doubled
    for slack as half an ulp would do) plus the worst-case FP32 accumulation
    over ``bk`` terms."""
    ulp_scale, tiny = (2.0**-10, 2.0**-14) if P.dtype == torch.float16 else (2.0**-7, 2.0**-126)
    Rt64 = Rt[:, :, :bk].double()
    for i in rows:
        a = L[:, i, :bk].double()
        exact = torch.einsum("rk,rnk->rn", a, Rt64)
        magnitude = torch.einsum("rk,rnk->rn", a.abs(), Rt64.abs())
        got = P[:, i, :bn].double()
        ulp = torch.clamp(exact.abs(), min=tiny) * ulp_scale
        assert torch.all((got - exact).abs() <= ulp + (bk + 2) * 2.0**-23 * magnitude)


def test_rank343_full_size_stages_match_oracle_on_sampled_positions():
    """Rank-343 FP16 square product at 16384^3 (the plain-mm API: ``B[K, N]``
    through the K x N right transform), the same sampled checks; the
    tensor-core reconstruct is held to one FP16 ulp of the oracle's
    ascending-order sum."""
    M = K = N = 16384
    s_ = 8
    A, B = randn_fp16((M, K), 0), randn_fp16((K, N), 1)
    shape = MatrixShape.from_dimensions(M, K, N, s_)
    bm, bk, bn = shape.block_rows, shape.block_inner, shape.block_columns
    dev = torch.device("cuda")
    Ad, Bd = A.to(dev), B.to(dev)
    L = torch.empty((343, bm, shape.inner_pitch), device=dev, dtype=torch.float16)
    Rt = torch.empty((343, bn, shape.inner_pitch), device=dev, dtype=torch.float16)
    P = torch.empty((343, bm, shape.column_pitch), device=dev, dtype=torch.float16)
    C = torch.empty((M, N), device=dev, dtype=torch.float16)
    _native.transform_a("rank343", Ad, L)
    _native.transform_b("rank343", Bd, Rt)
    _native.leaf_gemm(343, L, Rt, bm, bn, bk, P)
    _native.reconstruct("rank343", P, M, N, None, C)
    torch.cuda.synchronize()

    for i in _sample(bm, 4, seed=1):
        ref = oracle.left_transform("rank343", f32(_block_rows(A, s_, bm, i)))
        np.testing.assert_array_equal(_bits(L[:, i, :bk]), ref[:, 0, :].view(np.int16))
    for j in _sample(bn, 4, seed=2):
        cols = [p * bn + j for p in range(s_)]
        ref = oracle.right_transform("rank343", f32(B[:, cols]))  # [343, bk, 1]
        np.testing.assert_array_equal(_bits(Rt[:, j, :bk]), ref[:, :, 0].view(np.int16))

    _leaf_rows_within_bound(L, Rt, P, _sample(bm, 2, seed=3), bk, bn)

    # |C_o - ref| <= one FP16 ulp + the FP32 accumulation bound of the 343-term
    # +-1 sum (the tensor core adds in its own order; where the sum cancels,
    # that bound exceeds an ulp of the small result)
    W = np.abs(oracle.output_coefficients("rank343")).astype(np.float64)  # [64, 343]
    for i in _sample(bm, 4, seed=4):
        rows = [p * bm + i for p in range(s_)]
        products = P[:, i:i + 1, :bn].cpu().numpy()
        ref = oracle.output_transform("rank343", products, s_, N, None, "fp16").astype(np.float16)
        magnitude = (W @ np.abs(products[:, 0, :].astype(np.float64)))  # [64, bn], output o = (br, bc)
        bound_mag = magnitude.reshape(s_, s_, bn).reshape(s_, s_ * bn)  # row br, column bc * bn + c
        got = C[rows].cpu().numpy()
        ulp = np.spacing(np.abs(ref)).astype(np.float64)
        err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        assert np.all(err <= ulp + 345 * 2.0**-24 * bound_mag)
        assert np.mean(got == ref) > 0.99
    assert torch.isfinite(C).all()

    plan = Rank343Plan(M, K, N, dev)
    del L, Rt, P
    dynamic = plan.run(Ad, Bd, plan.allocate_workspace(0.9))
    assert torch.equal(dynamic.view(torch.int16), C.view(torch.int16))
    del dynamic
    packed = plan.run_packed(Ad, plan.pack_right(Bd, 0.9), plan.allocate_workspace(0.9, prepacked_right=True))
    assert torch.equal(packed.view(torch.int16), C.view(torch.int16))
