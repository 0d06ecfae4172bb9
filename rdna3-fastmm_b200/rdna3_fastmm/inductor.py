"""``torch.compile`` backend ``"rdna3-fastmm"`` (reference ``inductor.py:1-49``).

``compile_backend(gm, example_inputs, *, mode=None, options=None)`` rewrites
eligible BF16 linears to the ``rdna3_fastmm`` operators when gradients are
off and the runtime is the tested B200 stack, registers the external-matmul
callable, and hands the graph to Inductor.  Registered under the same name as
the reference's entry point (``pyproject.toml`` ``torch_dynamo_backends``).
"""

from __future__ import annotations

from typing import Any, Protocol, Sequence

import torch
import torch._inductor
import torch._inductor.config
from torch.fx import GraphModule

from .external_mm import rdna3_rank49_dynamic_v1_out
from .linear import rewrite_eligible_linears
from .runtime import is_tested_runtime


class CompiledGraph(Protocol):
    def __call__(self, *inputs: torch.Tensor) -> tuple[torch.Tensor, ...]: ...


def _enable_external_matmul() -> bool:
    if torch.is_grad_enabled() or torch.version.cuda is None or not torch.cuda.is_available():
        return False
    return is_tested_runtime(torch.device("cuda", torch.cuda.current_device()))


def compile_backend(graph_module: GraphModule, example_inputs: Sequence[torch.Tensor], *,
                    mode: str | None = None, options: dict[str, Any] | None = None) -> CompiledGraph:
    # ``list_mode_options(None)`` returns the table of every mode, not the
    # default mode's options; resolve None to "default" first
    inductor_options = dict(torch._inductor.list_mode_options(mode or "default"))
    inductor_options.update(options or {})
    if _enable_external_matmul():
        rewrite_eligible_linears(graph_module, list(example_inputs))
        configured = inductor_options.get("external_matmul", torch._inductor.config.external_matmul)
        choices = list(configured)
        if rdna3_rank49_dynamic_v1_out not in choices:
            choices.append(rdna3_rank49_dynamic_v1_out)
        inductor_options["external_matmul"] = choices
        inductor_options["max_autotune_gemm"] = True
        inductor_options["triton.cudagraphs"] = False
    return torch._inductor.compile(graph_module, list(example_inputs), options=inductor_options)


def register() -> None:
    """Make ``torch.compile(..., backend="rdna3-fastmm")`` work without an
    installed entry point."""
    from torch._dynamo import list_backends, register_backend

    if "rdna3-fastmm" not in list_backends(exclude_tags=()):
        register_backend(compile_backend, name="rdna3-fastmm")


register()
