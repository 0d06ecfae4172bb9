"""fmm_linear_noalloc: the linear for callers that cannot allocate device memory.

Some callers only receive device buffers (A, weight, bias, C) from a host
application that owns and budgets all device memory, or run in a loop that must
never call cudaMalloc because cudaMalloc can synchronise the device.  For them
``fmm_linear_noalloc`` keeps its transform and product planes in one fixed
32 MiB array inside the library instead of caller-provided planes.

These tests call it through the C ABI and compare it with ``fmm_linear`` fed
with caller planes, on two calls in a row (the second call reuses the array the
first one left behind), within the relative-L2 tolerance of the other linear
tests; they also check that a shape whose planes do not fit is refused.  The
file is named so that pytest collects it last.
"""

import pytest
import torch

from inputs import make_linear_inputs
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu

PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
TOLERANCE = 5e-3  # relative L2, as in the other linear tests


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


def _relative_l2(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b))


@pytest.mark.parametrize("name", list(PLANS))
def test_noalloc_matches_caller_planes_on_consecutive_calls(name):
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cases = [((257, 263, 269), 0, True), ((384, 512, 640), 10, False)]
    for (M, K, N), seed, with_bias in cases:  # two calls in a row
        A, W, bias = (t.to(device) if t is not None else None
                      for t in make_linear_inputs(M, K, N, seed=seed, bias=with_bias))
        expected = _with_caller_planes(name, A, W, bias)
        C = torch.full((M, N), float("nan"), device=device, dtype=torch.bfloat16)
        rc = _native.linear_noalloc(name, A, W, bias, C)
        assert rc == _native.FMM_OK, _native.last_error()
        torch.cuda.synchronize(device)
        assert torch.isfinite(C).all()
        assert _relative_l2(C, expected) < TOLERANCE


def test_noalloc_refuses_shapes_beyond_its_scratch():
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    M = K = N = 2048  # rank-7 planes: 3 x 7 x 1024 x 1024 x 2 B = 44 MiB > 32 MiB
    A, W, _ = (t.to(device) if t is not None else None for t in make_linear_inputs(M, K, N))
    C = torch.zeros((M, N), device=device, dtype=torch.bfloat16)
    rc = _native.linear_noalloc("rank7", A, W, None, C)
    assert rc == _native.FMM_ERR_TOO_LARGE
    assert "fmm_linear_noalloc" in _native.last_error()
    torch.cuda.synchronize(device)
    assert torch.count_nonzero(C) == 0  # nothing was launched
