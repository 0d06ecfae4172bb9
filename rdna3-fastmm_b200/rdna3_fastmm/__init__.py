"""B200-native fast matrix multiplication for BF16 ``F.linear``.

Drop-in for the operator surface of chelokot/rdna3-fastmm
(``src/rdna3_fastmm/__init__.py:1-5``): the same package name, plan classes,
``torch.library`` operators and ``torch.compile`` backend, executed by
hand-written sm_100a CUDA kernels behind a C ABI (``libfmm_sm100.so``).
"""

from rdna3_fastmm.certificate import ExpandedScheme, load_expanded_scheme

__version__ = "0.1.0"

__all__ = ["ExpandedScheme", "__version__", "load_expanded_scheme"]
