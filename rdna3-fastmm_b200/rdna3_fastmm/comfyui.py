"""ComfyUI model-patch node that compiles the diffusion model with this backend.

Drop-in for ``src/rdna3_fastmm/comfyui.py`` of chelokot/rdna3-fastmm (node
``:81-117``, guard filter ``:36-39``, runtime check ``:42-53``, ComfyUI helper
loader ``:61-73``): same node class name (``RDNA3FastMMCompile``, so saved
workflows keep working), one ``MODEL`` in and out.  The node clones the model
with ``disable_dynamic=True`` and installs ``compile_backend`` on its
``diffusion_model`` through ComfyUI's ``set_torch_compile_wrapper``; the
backend then rewrites the BF16 linears whose shapes the B200 dispatch tables
admit and leaves everything else to Inductor.  Static graphs only: dispatch is
decided on concrete dimensions.  Nothing is prepacked or retained, so
ComfyUI's cloning, patching and offloading see ordinary parameters.
"""

from __future__ import annotations

import logging
import sys
from importlib import import_module
from typing import Callable, Protocol, Sequence

BackendCompiler = Callable[..., object]
logger = logging.getLogger(__name__)

SUPPORTED_PYTHON = ((3, 12), (3, 14))  # [low, high)
REQUIRED_COMFYUI = "0.19.0"


class ComfyModel(Protocol):
    def clone(self, disable_dynamic: bool = False) -> "ComfyModel": ...


class GuardEntry(Protocol):
    name: str


def skip_comfy_transformer_option_guards(guard_entries: Sequence[GuardEntry]) -> list[bool]:
    """Dynamo guard filter: drop guards on ComfyUI's per-call
    ``transformer_options`` dict, which changes every sampling step and
    would otherwise force a recompile."""
    return ["transformer_options" not in entry.name for entry in guard_entries]


def _unsupported_reason() -> str | None:
    low, high = SUPPORTED_PYTHON
    if not low <= tuple(sys.version_info[:2]) < high:
        return "RDNA3 FastMM compilation requires Python 3.12 or 3.13"
    try:
        runtime = import_module("rdna3_fastmm.runtime")
    except ModuleNotFoundError as error:
        return f"missing Python dependency {error.name}"
    return runtime.unsupported_runtime_reason()


def _load_compile_backend() -> BackendCompiler:
    return import_module("rdna3_fastmm.inductor").compile_backend


def _load_compile_setter() -> Callable[..., None]:
    try:
        helpers = import_module("comfy_api.torch_helpers")
    except ModuleNotFoundError as error:
        if error.name is not None and error.name.startswith("comfy_api"):
            raise RuntimeError(f"RDNA3 FastMM requires ComfyUI {REQUIRED_COMFYUI} or newer") from error
        raise
    return helpers.set_torch_compile_wrapper


class RDNA3FastMMCompile:
    RETURN_TYPES = ("MODEL",)
    RETURN_NAMES = ("model",)
    FUNCTION = "compile_model"
    CATEGORY = "model_patches/compile"
    DESCRIPTION = (
        "Compiles the diffusion model with the B200 FastMM backend. BF16 Linear shapes "
        "measured to win on B200 use reduced-multiplication kernels; all other operations "
        "remain ordinary PyTorch Inductor operations."
    )
    EXPERIMENTAL = True

    @classmethod
    def INPUT_TYPES(cls) -> dict:
        return {"required": {"model": ("MODEL",)}}

    def compile_model(self, model: ComfyModel) -> tuple[ComfyModel]:
        reason = _unsupported_reason()
        if reason is not None:
            raise RuntimeError(f"Cannot enable RDNA3 FastMM: {reason}")
        set_compile_wrapper = _load_compile_setter()
        backend = _load_compile_backend()
        patched = model.clone(disable_dynamic=True)
        set_compile_wrapper(
            model=patched,
            backend=backend,
            options={"guard_filter_fn": skip_comfy_transformer_option_guards},
            dynamic=False,
            keys=["diffusion_model"],
        )
        logger.info("Enabled RDNA3 FastMM (B200) for the ComfyUI diffusion model")
        return (patched,)


NODE_CLASS_MAPPINGS = {"RDNA3FastMMCompile": RDNA3FastMMCompile}
NODE_DISPLAY_NAME_MAPPINGS = {"RDNA3FastMMCompile": "RDNA3 FastMM Compile"}
