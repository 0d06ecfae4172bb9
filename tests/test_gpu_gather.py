"""The gathering reconstruct (``fmm_reconstruct_gather``) on one B200.

A row-sharded linear stores each rank's output rows into every rank's gather
buffer at once.  On one GPU the destinations are separate local buffers; the
kernels cannot tell them from peer mappings.  Every destination must hold
exactly ``fmm_reconstruct``'s bits (bias included), and no byte outside the
``M x N`` region of each destination may change (padding columns of a wider
``ldc`` and guard rows after the last row stay NaN).

Rank 48/49 with 16-byte-aligned rows (bn, N, ldc multiples of 8) run the
staged kernel whose bulk copies write the destinations.  Other shapes, and
rank 7, run the register kernel with per-element stores.  A small SM budget
gives the staged kernel many tiles per CTA, so both of its staging buffers are
reused many times.
"""

import numpy as np
import pytest
import torch

from inputs import make_linear_inputs, random_products
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu

PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
# (M, N): 16-byte-aligned rows with ragged edges (staged bulk copies for rank
# 48/49); odd N (register kernel); c5b's shape per GPU at 8 GPUs, cut to 2048 rows
SHAPES = [(1029, 2064), (2048, 12288), (257, 269), (130, 514)]
GUARD_ROWS = 2


def _products(name: str, M: int, N: int, planes=torch.float16):
    plan = PLANS[name]
    s = MatrixShape.from_dimensions(M, 64, N, plan.scheme_size)
    P = torch.zeros((plan.rank, s.block_rows, s.column_pitch), device="cuda", dtype=planes)
    P[:, :, : s.block_columns] = random_products(plan.rank, s.block_rows, s.block_columns, seed=5).to(planes).cuda()
    return P


def _check(name, M, N, P, bias, ndest, ldc):
    expected = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    _native.reconstruct(name, P, M, N, bias, expected)
    dests = [torch.full(((M + GUARD_ROWS) * ldc,), float("nan"), device="cuda", dtype=torch.bfloat16)
             for _ in range(ndest)]
    _native.reconstruct_gather(name, P, M, N, bias, [d.data_ptr() for d in dests], ldc, torch.bfloat16)
    torch.cuda.synchronize()
    want = expected.view(torch.int16)
    for d in dests:
        rows = d[: M * ldc].view(M, ldc)
        assert torch.equal(rows[:, :N].view(torch.int16), want)
        assert torch.isnan(rows[:, N:].float()).all()
        assert torch.isnan(d[M * ldc:].float()).all()


@pytest.mark.parametrize("name", list(PLANS))
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("ndest", [1, 3, 8])
def test_gather_writes_reconstruct_bits_into_every_destination(name, shape, with_bias, ndest):
    M, N = shape
    _, _, bias = make_linear_inputs(M, 8, N, seed=1, bias=True)
    P = _products(name, M, N)
    _check(name, M, N, P, bias.cuda() if with_bias else None, ndest, N)


@pytest.mark.parametrize("name", ["rank48", "rank49"])
@pytest.mark.parametrize("sms", [2, 16])
def test_staged_gather_under_a_small_sm_budget(name, sms):
    """A few CTAs each take many tiles: the staging buffers alternate and the
    copies of earlier tiles are still in flight while later tiles compute."""
    M, N = 2048, 12288
    P = _products(name, M, N)
    _native.set_sm_budget(sms)
    try:
        _check(name, M, N, P, None, 8, N)
    finally:
        _native.set_sm_budget(0)


@pytest.mark.parametrize("name", ["rank48", "rank49"])
def test_gather_with_a_padded_leading_dimension(name):
    """ldc > N (a multiple of 8, so still the staged kernel): the padding
    columns between rows are never written."""
    M, N = 1029, 2064
    _, _, bias = make_linear_inputs(M, 8, N, seed=2, bias=True)
    P = _products(name, M, N)
    _check(name, M, N, P, bias.cuda(), 4, N + 24)


def test_gather_with_bf16_planes():
    """Rank 49 with BF16 planes (the (bfloat16, bfloat16) precision pair)."""
    M, N = 1029, 2064
    P = _products("rank49", M, N, planes=torch.bfloat16)
    _check("rank49", M, N, P, None, 3, N)


def test_gather_with_an_unaligned_destination_uses_element_stores():
    """A destination off the 16-byte grid takes the register kernel; its bits
    are the same."""
    M, N = 1029, 2064
    P = _products("rank48", M, N)
    expected = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    _native.reconstruct("rank48", P, M, N, None, expected)
    store = torch.full((M * N + 8,), float("nan"), device="cuda", dtype=torch.bfloat16)
    aligned = torch.full((M * N,), float("nan"), device="cuda", dtype=torch.bfloat16)
    _native.reconstruct_gather("rank48", P, M, N, None, [aligned.data_ptr(), store[1:].data_ptr()], N,
                               torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(aligned.view(M, N).view(torch.int16), expected.view(torch.int16))
    assert torch.equal(store[1:M * N + 1].view(M, N).view(torch.int16), expected.view(torch.int16))
    assert torch.isnan(store[0].float()) and torch.isnan(store[M * N + 1:].float()).all()
    assert np.isfinite(expected.float().cpu().numpy()).all()
