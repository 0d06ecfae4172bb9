"""fmm_linear_noalloc: the linear for callers that cannot allocate device memory.

Some callers only receive device buffers (A, weight, bias, C) from a host
application that owns and budgets all device memory, or run in a loop that must
never call cudaMalloc because cudaMalloc can synchronise the device.  For them
``fmm_linear_noalloc`` keeps its transform and product planes in one fixed
32 MiB array inside the library instead of caller-provided planes.

These tests call it through the C ABI, several calls in a row per scheme (each
later call runs on what the earlier ones left in the array, the largest call
first, so a smaller ragged call must rewrite every plane element it reads),
and require:

* bitwise equality with ``fmm_linear`` fed with caller planes -- the same
  kernels run in the same order, so any difference is a scratch-layout bug;
* agreement with the CPU oracle within the reference's relative-L2 tolerance;
* a shape whose planes fill the array exactly is accepted, one 256 bytes
  larger is refused and launches nothing.

The file is named so that pytest collects it last.
"""

import numpy as np
import pytest
import torch

from inputs import f32, make_linear_inputs
from oracle import fmm_oracle as oracle
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu

PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
TOLERANCE = 5e-3  # relative L2 against the oracle, as in the other linear tests
SCRATCH_BYTES = 32 << 20  # FMM_NOALLOC_SCRATCH_BYTES

# calls in order: (M, K, N), seed, bias.  The first call of rank 7 and of
# rank 49 needs exactly SCRATCH_BYTES of planes; ragged shapes follow.
CALLS = {
    "rank7": [((240, 2672, 3072), 0, False), ((257, 263, 269), 3, True), ((384, 512, 640), 10, False)],
    "rank48": [((1024, 1024, 1024), 0, True), ((257, 263, 269), 3, True), ((130, 1030, 514), 10, False)],
    "rank49": [((292, 736, 5120), 0, False), ((257, 263, 269), 3, True), ((130, 1030, 514), 10, True)],
}


def _scratch_bytes(name, M, K, N):
    d = _native.plan_dims(name, M, K, N)
    up = lambda n: -(-n // 256) * 256  # noqa: E731
    return up(d.left_elements * 2) + up(d.right_elements * 2) + up(d.product_elements * 2)


def _with_caller_planes(name, A, W, bias):
    plan_type = PLANS[name]
    M, K = A.shape
    N = W.shape[0]
    s = MatrixShape.from_dimensions(M, K, N, plan_type.scheme_size)
    L = torch.empty((plan_type.rank, s.block_rows, s.inner_pitch), device=A.device, dtype=torch.float16)
    Rt = torch.empty((plan_type.rank, s.block_columns, s.inner_pitch), device=A.device, dtype=torch.float16)
    P = torch.empty((plan_type.rank, s.block_rows, s.column_pitch), device=A.device, dtype=torch.float16)
    C = torch.empty((M, N), device=A.device, dtype=torch.bfloat16)
    _native.linear(name, A, W, bias, C, L, Rt, P, prepacked=False)
    return C


def test_boundary_shapes_fill_the_scratch_exactly():
    assert _scratch_bytes("rank7", 240, 2672, 3072) == SCRATCH_BYTES
    assert _scratch_bytes("rank49", 292, 736, 5120) == SCRATCH_BYTES
    assert _scratch_bytes("rank7", 166, 2704, 3184) == SCRATCH_BYTES + 256


@pytest.mark.parametrize("name", list(PLANS))
def test_noalloc_equals_caller_planes_bitwise_on_consecutive_calls(name):
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    for (M, K, N), seed, with_bias in CALLS[name]:
        assert _scratch_bytes(name, M, K, N) <= SCRATCH_BYTES
        A_h, W_h, b_h = make_linear_inputs(M, K, N, seed=seed, bias=with_bias)
        A, W = A_h.to(device), W_h.to(device)
        bias = b_h.to(device) if b_h is not None else None
        expected = _with_caller_planes(name, A, W, bias)
        C = torch.full((M, N), float("nan"), device=device, dtype=torch.bfloat16)
        rc = _native.linear_noalloc(name, A, W, bias, C)
        assert rc == _native.FMM_OK, _native.last_error()
        torch.cuda.synchronize(device)
        assert torch.equal(C.view(torch.int16), expected.view(torch.int16)), (name, M, K, N)
        ref = oracle.linear(name, f32(A_h), f32(W_h), f32(b_h) if b_h is not None else None)
        got = C.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert oracle.relative_l2(got, ref) < TOLERANCE


def test_noalloc_refuses_shapes_beyond_its_scratch():
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    for M, K, N in [(166, 2704, 3184), (2048, 2048, 2048)]:  # 256 B over; 44 MiB
        A, W, _ = (t.to(device) if t is not None else None for t in make_linear_inputs(M, K, N))
        C = torch.zeros((M, N), device=device, dtype=torch.bfloat16)
        rc = _native.linear_noalloc("rank7", A, W, None, C)
        assert rc == _native.FMM_ERR_TOO_LARGE
        assert "fmm_linear_noalloc" in _native.last_error()
        torch.cuda.synchronize(device)
        assert torch.count_nonzero(C) == 0  # nothing was launched
