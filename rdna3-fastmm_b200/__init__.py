"""ComfyUI custom-node entry point: copy or link this directory into
``ComfyUI/custom_nodes/``.

Loads the ``rdna3_fastmm`` package that sits beside this file (reference
entry point: the repository-root ``__init__.py`` of chelokot/rdna3-fastmm) and
refuses to run next to a different, already imported ``rdna3_fastmm``.
"""

import sys
from pathlib import Path

_here = Path(__file__).resolve().parent
_loaded = sys.modules.get("rdna3_fastmm")
if _loaded is not None:
    _file = getattr(_loaded, "__file__", None)
    if _file is None or _here not in Path(_file).resolve().parents:
        raise RuntimeError(
            "A different rdna3_fastmm package is already loaded; restart ComfyUI "
            "after removing the conflicting installation"
        )

sys.path.insert(0, str(_here))
try:
    from rdna3_fastmm.comfyui import NODE_CLASS_MAPPINGS, NODE_DISPLAY_NAME_MAPPINGS
finally:
    sys.path.remove(str(_here))

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
