"""The reference-side ctypes binding runs the reference's ``_LinearPlan``
launch sequence on B200 (``src/rdna3_fastmm/runtime.py:700-777`` of
chelokot/rdna3-fastmm: left transform, weight transform, ``torch.bmm`` into the
products, output transform with or without bias).  The plan below restates
that sequence with the stub's ``B200Launches`` in place of the Triton
launches; its output must match the CPU oracle within the reference's 5e-3
relative-L2 tolerance and equal the package's own ``run_linear`` /
``run_linear_packed`` bit for bit (the same kernels run in the same order)."""

import numpy as np
import pytest
import torch

from inputs import f32, make_linear_inputs
from oracle import fmm_oracle as oracle
from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan
from test_reference_binding_cpu import load_binding

pytestmark = pytest.mark.gpu

PLANS = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}


def make_reference_style_plan(binding, name, M, K, N, planes=torch.float16):
    scheme_size = PLANS[name].scheme_size

    class Plan(binding.B200Launches):
        rank = PLANS[name].rank
        shape = MatrixShape.from_dimensions(M, K, N, scheme_size)

        def workspace(self, device, prepacked: bool):
            shapes = binding.plane_shapes(self.rank, M, K, N)
            return {k: torch.empty(v, device=device, dtype=planes) for k, v in shapes.items()
                    if not (prepacked and k == "right")}

        def run_linear(self, x, weight, ws, bias, out):  # runtime.py:700-741
            self._transform_left(x, ws["left"])
            self._transform_weight(weight, ws["right"])
            self._products(ws["left"], ws["right"], ws["products"])
            if bias is None:
                self._reconstruct(ws["products"], out)
            else:
                self._reconstruct_bias(ws["products"], bias, out)
            return out

        def run_linear_packed(self, x, packed, ws, bias, out):  # runtime.py:743-777
            self._transform_left(x, ws["left"])
            self._products(ws["left"], packed, ws["products"])
            if bias is None:
                self._reconstruct(ws["products"], out)
            else:
                self._reconstruct_bias(ws["products"], bias, out)
            return out

    return Plan()


@pytest.mark.parametrize("name", list(PLANS))
@pytest.mark.parametrize("shape", [(257, 263, 269), (512, 1024, 1024)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("with_bias", [False, True])
def test_reference_launch_sequence_through_the_binding(name, shape, with_bias):
    binding = load_binding()
    binding._lib = binding.load(str(_native.LIBRARY_PATH))
    M, K, N = shape
    device = torch.device("cuda", 0)
    A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=with_bias)
    Ad, Wd = A.to(device), W.to(device)
    bd = bias.to(device) if bias is not None else None
    plan = make_reference_style_plan(binding, name, M, K, N)

    out = torch.empty((M, N), device=device, dtype=torch.bfloat16)
    plan.run_linear(Ad, Wd, plan.workspace(device, False), bd, out)
    packed = torch.empty(binding.plane_shapes(plan.rank, M, K, N)["right"], device=device, dtype=torch.float16)
    plan._transform_weight(Wd, packed)
    out_packed = torch.empty_like(out)
    plan.run_linear_packed(Ad, packed, plan.workspace(device, True), bd, out_packed)
    torch.cuda.synchronize(device)

    ref = oracle.linear(name, f32(A), f32(W), f32(bias) if bias is not None else None)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.relative_l2(got, ref) < 5e-3
    assert torch.equal(out.view(torch.int16), out_packed.view(torch.int16))

    own = PLANS[name](M, K, N, device, dtype=torch.bfloat16, compute_dtype=torch.float16)
    expected = own.run_linear(Ad, Wd, own.allocate_workspace(0.5), bd)
    torch.cuda.synchronize(device)
    assert torch.equal(out.view(torch.int16), expected.view(torch.int16))


@pytest.mark.parametrize("with_bias", [False, True])
def test_reference_launch_sequence_with_bf16_planes(with_bias):
    """Rank49Plan's (bfloat16, bfloat16) pair through the binding: BF16 planes
    and products, the BF16 leaf GEMM entry point."""
    binding = load_binding()
    binding._lib = binding.load(str(_native.LIBRARY_PATH))
    M, K, N = 257, 263, 269
    device = torch.device("cuda", 0)
    A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=with_bias)
    Ad, Wd = A.to(device), W.to(device)
    bd = bias.to(device) if bias is not None else None
    plan = make_reference_style_plan(binding, "rank49", M, K, N, planes=torch.bfloat16)
    out = torch.empty((M, N), device=device, dtype=torch.bfloat16)
    plan.run_linear(Ad, Wd, plan.workspace(device, False), bd, out)
    own = Rank49Plan(M, K, N, device, dtype=torch.bfloat16, compute_dtype=torch.bfloat16)
    expected = own.run_linear(Ad, Wd, own.allocate_workspace(0.5), bd)
    torch.cuda.synchronize(device)
    assert torch.equal(out.view(torch.int16), expected.view(torch.int16))
    ref = oracle.linear("rank49", f32(A), f32(W), f32(bias) if bias is not None else None, planes="bf16")
    assert oracle.relative_l2(out.float().cpu().numpy(), ref) < 2e-3
