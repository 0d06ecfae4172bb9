"""Inductor ``external_matmul`` callable (the reference's
``src/rdna3_fastmm/external_mm.py``).

Inductor's GEMM autotuner may call ``rdna3_rank49_dynamic_v1_out(left, right,
*, out)`` for any ``mm`` it lowers.  The callable asks the rank-49 plan
itself whether it takes the call, instead of restating the plan's rules:

1. the plan's gate (``Rank49Plan.is_recommended``: FP16 operands and FP16
   leaves, a shape in the plan's measured ``dynamic_shapes`` table, the
   tested runtime) decides whether the shape goes to the B200 kernels at all;
2. constructing the plan and ``plan.run`` validate device, dtype, layout,
   autograd and storage overlap, raising ``ValueError`` before any launch;
3. ``allocate_workspace`` raises ``MemoryError`` when the planes do not fit
   in free device memory.

Whatever the plan refuses (and every call with autograd recording) becomes
``torch.mm(left, right, out=out)``.  No plain-mm shape beats cuBLAS on B200,
so the measured table is empty and every call is the library product.
"""

from __future__ import annotations

import torch

from .runtime import Rank49Plan

__all__ = ["is_rank49_dynamic_eligible", "rdna3_rank49_dynamic_v1_out"]


def _plan_for(left: torch.Tensor, right: torch.Tensor) -> Rank49Plan | None:
    """A rank-49 plan for ``left @ right`` when the plan's gate admits it."""
    if torch.is_grad_enabled() or left.dim() != 2 or right.dim() != 2:
        return None
    shape = (left.shape[0], left.shape[1], right.shape[1])
    if shape not in Rank49Plan.dynamic_shapes:  # cheap first: no plan for unmeasured shapes
        return None
    try:
        plan = Rank49Plan(*shape, left.device, left.dtype)
    except ValueError:  # not a CUDA device, or a precision pair the plan lacks
        return None
    return plan if plan.is_recommended() else None


def _validated(plan: Rank49Plan, left: torch.Tensor, right: torch.Tensor, out: torch.Tensor) -> bool:
    try:
        plan._validate_left(left)
        plan._validate_right(right)
        plan._output(out)
        plan._validate_output_storage(out, left, right)
    except ValueError:
        return False
    return True


def is_rank49_dynamic_eligible(left: torch.Tensor, right: torch.Tensor, out: torch.Tensor) -> bool:
    """Whether ``rdna3_rank49_dynamic_v1_out`` runs the B200 plan for these
    tensors (memory permitting)."""
    plan = _plan_for(left, right)
    return plan is not None and _validated(plan, left, right, out)


def rdna3_rank49_dynamic_v1_out(left: torch.Tensor, right: torch.Tensor, *, out: torch.Tensor) -> None:
    plan = _plan_for(left, right)
    if plan is not None and _validated(plan, left, right, out):
        try:
            workspace = plan.allocate_workspace(max_free_memory_fraction=1.0)
        except MemoryError:
            workspace = None
        if workspace is not None:
            plan.run(left, right, workspace, out)
            return
    torch.mm(left, right, out=out)
