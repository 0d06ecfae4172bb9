"""``torch.library`` operators and the FX rewrite that selects them.

Drop-in for ``src/rdna3_fastmm/linear.py`` of chelokot/rdna3-fastmm:

* ``torch.ops.rdna3_fastmm.linear`` (rank 49) and
  ``torch.ops.rdna3_fastmm.linear_rank7`` -- allocating ``F.linear``
  contract ``(input[..., K], weight[N, K], bias[N] | None) -> [..., N]``,
  ``mutates_args={}`` (reference ``linear.py:50-167``);
  ``torch.ops.rdna3_fastmm.linear_rank48`` is the rank-48 twin;
* ``rewrite_eligible_linears`` / ``_linear_node_target``: replace an
  ``aten.linear`` node by one of the operators only when the plan's measured
  B200 dispatch table admits the shape and the call's allocations fit in half
  of the free device memory (reference ``linear.py:175-288``).

The operators allocate their planes per call, free the transformed inputs
before the output is allocated (as the reference does, ``linear.py:116-120``),
and run every stage on the current stream through ``libfmm_sm100.so``.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
from torch.fx import GraphModule, Node
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.passes.fake_tensor_prop import FakeTensorProp

from . import _native
from .runtime import MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan, _LinearPlan

LINEAR_TARGETS = frozenset({torch._C._nn.linear, torch.ops.aten.linear.default})
MAX_LINEAR_ALLOCATION_FREE_FRACTION = 0.5


def _run_linear(plan_type: type[_LinearPlan], input_tensor: torch.Tensor, weight: torch.Tensor,
                bias: Optional[torch.Tensor]) -> torch.Tensor:
    inner = input_tensor.shape[-1]
    columns = weight.shape[0]
    flat = input_tensor.reshape(-1, inner).contiguous()
    weight = weight.contiguous()
    rows = flat.shape[0]
    device = input_tensor.device
    shape = MatrixShape.from_dimensions(rows, inner, columns, plan_type.scheme_size)
    rank = plan_type.rank
    half = torch.float16
    with torch.cuda.device(device):
        left = torch.empty((rank, shape.block_rows, shape.inner_pitch), device=device, dtype=half)
        right = torch.empty((rank, shape.block_columns, shape.inner_pitch), device=device, dtype=half)
        _native.transform_a(plan_type.scheme, flat, left)
        _native.transform_w(plan_type.scheme, weight, right)
        products = torch.empty((rank, shape.block_rows, shape.column_pitch), device=device, dtype=half)
        _native.leaf_gemm(rank, left, right, shape.block_rows, shape.block_columns, shape.block_inner,
                          products)
        del left, right
        out = torch.empty((rows, columns), device=device, dtype=input_tensor.dtype)
        _native.reconstruct(plan_type.scheme, products, rows, columns,
                            None if bias is None else bias.contiguous(), out)
    return out.reshape(*input_tensor.shape[:-1], columns)


def _check_operands(input_tensor: torch.Tensor, weight: torch.Tensor,
                    bias: Optional[torch.Tensor]) -> None:
    if input_tensor.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != input_tensor.dtype:
        raise ValueError("rdna3_fastmm linear operators take BF16 or FP16 input and weight of one dtype")
    if bias is not None and bias.dtype != input_tensor.dtype:
        raise ValueError("rdna3_fastmm linear operators take a bias of the input's dtype")
    if weight.ndim != 2 or input_tensor.shape[-1] != weight.shape[1]:
        raise ValueError("input and weight shapes do not form a linear")
    if bias is not None and tuple(bias.shape) != (weight.shape[0],):
        raise ValueError("bias must have shape [N]")


def _create_linear_operator(name: str, plan_type: type[_LinearPlan]) -> Callable[..., torch.Tensor]:
    @torch.library.custom_op(name, mutates_args=(), device_types="cuda")
    def operator(input_tensor: torch.Tensor, weight: torch.Tensor,
                 bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        _check_operands(input_tensor, weight, bias)
        return _run_linear(plan_type, input_tensor, weight, bias)

    @operator.register_fake
    def _(input_tensor, weight, bias=None):
        return input_tensor.new_empty((*input_tensor.shape[:-1], weight.shape[0]))

    return operator


rdna3_linear = _create_linear_operator("rdna3_fastmm::linear", Rank49Plan)
rdna3_rank7_linear = _create_linear_operator("rdna3_fastmm::linear_rank7", Rank7Plan)
rdna3_rank48_linear = _create_linear_operator("rdna3_fastmm::linear_rank48", Rank48Plan)

RDNA3_LINEAR_OP = torch.ops.rdna3_fastmm.linear.default
RDNA3_RANK7_LINEAR_OP = torch.ops.rdna3_fastmm.linear_rank7.default
RDNA3_RANK48_LINEAR_OP = torch.ops.rdna3_fastmm.linear_rank48.default


def _node_tensor(node: Node) -> torch.Tensor | None:
    value = node.meta.get("val", node.meta.get("example_value"))
    return value if isinstance(value, torch.Tensor) else None


def _allocation_bytes(plan_type: type[_LinearPlan], shape: tuple[int, int, int]) -> int:
    rows, inner, columns = shape
    s = MatrixShape.from_dimensions(rows, inner, columns, plan_type.scheme_size)
    planes = plan_type.rank * (
        s.block_rows * s.inner_pitch + s.block_columns * s.inner_pitch + s.block_rows * s.column_pitch
    )
    return planes * torch.float16.itemsize + rows * columns * torch.bfloat16.itemsize


def _has_linear_memory_budget(plan_type: type[_LinearPlan], shape: tuple[int, int, int],
                              device: torch.device) -> bool:
    free, _ = torch.cuda.mem_get_info(device)
    return _allocation_bytes(plan_type, shape) <= free * MAX_LINEAR_ALLOCATION_FREE_FRACTION


_CANDIDATES = (
    (Rank7Plan, RDNA3_RANK7_LINEAR_OP),
    (Rank49Plan, RDNA3_LINEAR_OP),
    (Rank48Plan, RDNA3_RANK48_LINEAR_OP),
)


def _linear_node_target(node: Node):
    if node.op != "call_function" or node.target not in LINEAR_TARGETS:
        return None
    if node.kwargs or len(node.args) not in (2, 3):
        return None
    input_node, weight_node = node.args[:2]
    bias_node = node.args[2] if len(node.args) == 3 else None
    if not isinstance(input_node, Node) or not isinstance(weight_node, Node):
        return None
    x, w = _node_tensor(input_node), _node_tensor(weight_node)
    if x is None or w is None or x.ndim < 2 or w.ndim != 2:
        return None
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        return None
    if x.device.type != "cuda" or w.device != x.device:
        return None
    if not x.is_contiguous() or not w.is_contiguous():
        return None
    inner = x.shape[-1]
    columns, weight_inner = w.shape
    if inner != weight_inner:
        return None
    if not all(isinstance(d, int) for d in (*x.shape, columns)):
        return None
    has_bias = bias_node is not None
    if isinstance(bias_node, Node):
        b = _node_tensor(bias_node)
        if (b is None or tuple(b.shape) != (columns,) or b.dtype != torch.bfloat16
                or b.device != x.device or not b.is_contiguous()):
            return None
    elif bias_node is not None:
        return None
    rows = x.numel() // inner
    shape = (rows, inner, columns)
    for plan_type, target in _CANDIDATES:
        if plan_type.has_measured_linear_win(shape, has_bias=has_bias):
            return target if _has_linear_memory_budget(plan_type, shape, x.device) else None
    return None


def rewrite_eligible_linears(graph_module: GraphModule, example_inputs: list[torch.Tensor]) -> int:
    """Rewrite every eligible ``aten.linear`` node; returns how many."""
    nodes = tuple(n for n in graph_module.graph.nodes
                  if n.op == "call_function" and n.target in LINEAR_TARGETS)
    if any(isinstance(a, Node) and _node_tensor(a) is None for n in nodes for a in n.args):
        # parameters reached through get_attr are real tensors; let the fake
        # mode wrap them instead of refusing the graph
        FakeTensorProp(graph_module, FakeTensorMode(allow_non_fake_inputs=True)).propagate(*example_inputs)
    rewritten = 0
    for node in nodes:
        target = _linear_node_target(node)
        if target is None:
            continue
        input_node, weight_node = node.args[:2]
        bias_node = node.args[2] if len(node.args) == 3 else None
        with graph_module.graph.inserting_before(node):
            replacement = graph_module.graph.call_function(target, args=(input_node, weight_node, bias_node))
        replacement.meta = node.meta.copy()
        node.replace_all_uses_with(replacement)
        graph_module.graph.erase_node(node)
        rewritten += 1
    if rewritten:
        graph_module.graph.lint()
        graph_module.recompile()
    return rewritten
