"""The binding a maintainer of chelokot/rdna3-fastmm would add to run its plans
on B200 through ``libfmm_sm100.so`` (drop it into the reference tree as
``src/rdna3_fastmm/b200.py``).

The reference is Python, so its FFI is ctypes.  ``B200Launches`` replaces the
launch methods of the reference's ``_LinearPlan``
(``src/rdna3_fastmm/runtime.py``): ``_transform_left`` (:597-615),
``_transform_right`` (:617-635), ``_transform_weight`` (:637-655),
``_reconstruct`` / ``_reconstruct_bias`` (:657-698), and adds ``_products``
for the ``torch.bmm(L, Rw, out=P)`` calls of ``run_linear`` /
``run_linear_packed`` (:728-732, :768-772).  Mixed in ahead of ``_LinearPlan``
(``class Rank7Plan(B200Launches, _LinearPlan)``), every launch goes to the C
ABI declared in ``include/fmm_sm100.h`` on torch's current stream.

Plane buffers must use the library's layouts (``fmm_plan_dims``): rows padded
to ``ldk = round_up(bk, 8)`` / ``ldp = round_up(bn, 8)`` elements, and the
transformed right operand stored K-major as ``[rank, bn, ldk]`` (the transpose
of the reference's ``[rank, bk, bn]``); ``plane_shapes`` gives the three
shapes for a plan's workspace allocation.
"""

from __future__ import annotations

import ctypes
import os

import torch

FMM_OK = 0
FMM_DTYPE_BF16 = 0
FMM_DTYPE_F16 = 1
FMM_DTYPE_BF16_BF16 = 2


class FmmDims(ctypes.Structure):
    """``fmm_dims`` of include/fmm_sm100.h."""

    _fields_ = [(name, ctypes.c_int64) for name in (
        "scheme_size", "rank", "bm", "bk", "bn", "ldk", "ldp",
        "left_elements", "right_elements", "product_elements")]


_P, _I64, _INT = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int

# argument lists of the entry points this binding calls, in header order
ARGTYPES = {
    # int fmm_plan_dims(int scheme, int64_t M, int64_t K, int64_t N, fmm_dims* out)
    "fmm_plan_dims": [_INT, _I64, _I64, _I64, ctypes.POINTER(FmmDims)],
    # int fmm_transform_a(int scheme, int dtype, const void* A, int64_t M, int64_t K,
    #                     int64_t lda, void* L, fmm_stream_t stream)
    "fmm_transform_a": [_INT, _INT, _P, _I64, _I64, _I64, _P, _P],
    # int fmm_transform_w(int scheme, int dtype, const void* W, int64_t N, int64_t K,
    #                     int64_t ldw, void* Rt, fmm_stream_t stream)
    "fmm_transform_w": [_INT, _INT, _P, _I64, _I64, _I64, _P, _P],
    # int fmm_transform_b(int scheme, int dtype, const void* B, int64_t K, int64_t N,
    #                     int64_t ldb, void* Rt, fmm_stream_t stream)
    "fmm_transform_b": [_INT, _INT, _P, _I64, _I64, _I64, _P, _P],
    # int fmm_leaf_gemm(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn,
    #                   int64_t bk, void* P, fmm_stream_t stream)
    "fmm_leaf_gemm": [_INT, _P, _P, _I64, _I64, _I64, _P, _P],
    # int fmm_leaf_gemm_bf16(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn,
    #                        int64_t bk, void* P, fmm_stream_t stream)
    "fmm_leaf_gemm_bf16": [_INT, _P, _P, _I64, _I64, _I64, _P, _P],
    # int fmm_reconstruct(int scheme, int dtype, const void* P, int64_t M, int64_t N,
    #                     const void* bias, void* C, int64_t ldc, fmm_stream_t stream)
    "fmm_reconstruct": [_INT, _INT, _P, _I64, _I64, _P, _P, _I64, _P],
    # const char* fmm_last_error_string(void)
    "fmm_last_error_string": [],
}


def load(path: str | None = None) -> ctypes.CDLL:
    """Open the library (``FMM_SM100_LIBRARY`` or the loader's search path)
    and declare the entry points this binding uses."""
    lib = ctypes.CDLL(path or os.environ.get("FMM_SM100_LIBRARY", "libfmm_sm100.so"))
    for name, args in ARGTYPES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_char_p if name == "fmm_last_error_string" else ctypes.c_int
    return lib


_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != FMM_OK:
        raise RuntimeError(f"{what}: {library().fmm_last_error_string().decode()} (error {rc})")


def _dtype(tensor: torch.Tensor, planes: torch.Tensor) -> int:
    """Precision id: the operand (or output) type with the plane type -- the
    plan's ``(dtype, compute_dtype)`` pair."""
    pair = (tensor.dtype, planes.dtype)
    if pair == (torch.bfloat16, torch.float16):
        return FMM_DTYPE_BF16
    if pair == (torch.float16, torch.float16):
        return FMM_DTYPE_F16
    if pair == (torch.bfloat16, torch.bfloat16):
        return FMM_DTYPE_BF16_BF16
    raise ValueError(f"libfmm_sm100 does not take {tensor.dtype} operands with {planes.dtype} planes")


def _stream(tensor: torch.Tensor) -> int:
    return torch.cuda.current_stream(tensor.device).cuda_stream


def plane_shapes(rank: int, rows: int, inner: int, columns: int) -> dict:
    """Shapes of the left, right and product planes the library expects."""
    dims = FmmDims()
    _check(library().fmm_plan_dims(rank, rows, inner, columns, ctypes.byref(dims)), "fmm_plan_dims")
    return {"left": (rank, dims.bm, dims.ldk), "right": (rank, dims.bn, dims.ldk),
            "products": (rank, dims.bm, dims.ldp)}


class B200Launches:
    """Launch methods of ``_LinearPlan`` on the B200 library.  Uses the
    plan's ``rank`` (the scheme id: 7, 48, 49 or 343) and ``shape``."""

    def _transform_left(self, source: torch.Tensor, output: torch.Tensor) -> None:
        rows, inner = source.shape
        _check(library().fmm_transform_a(self.rank, _dtype(source, output), source.data_ptr(), rows, inner,
                                         source.stride(0), output.data_ptr(), _stream(source)),
               "fmm_transform_a")

    def _transform_right(self, source: torch.Tensor, output: torch.Tensor) -> None:
        inner, columns = source.shape
        _check(library().fmm_transform_b(self.rank, _dtype(source, output), source.data_ptr(), inner, columns,
                                         source.stride(0), output.data_ptr(), _stream(source)),
               "fmm_transform_b")

    def _transform_weight(self, source: torch.Tensor, output: torch.Tensor) -> None:
        columns, inner = source.shape
        _check(library().fmm_transform_w(self.rank, _dtype(source, output), source.data_ptr(), columns, inner,
                                         source.stride(0), output.data_ptr(), _stream(source)),
               "fmm_transform_w")

    def _products(self, left: torch.Tensor, right: torch.Tensor, products: torch.Tensor) -> None:
        """Replaces ``torch.bmm(left, right, out=products)`` (FP16 planes, or
        BF16 planes for the rank-49 ``(bfloat16, bfloat16)`` pair)."""
        s = self.shape
        gemm = library().fmm_leaf_gemm_bf16 if left.dtype == torch.bfloat16 else library().fmm_leaf_gemm
        _check(gemm(self.rank, left.data_ptr(), right.data_ptr(), s.block_rows, s.block_columns,
                    s.block_inner, products.data_ptr(), _stream(left)),
               "fmm_leaf_gemm")

    def _reconstruct(self, products: torch.Tensor, output: torch.Tensor) -> None:
        self._reconstruct_bias(products, None, output)

    def _reconstruct_bias(self, products: torch.Tensor, bias: torch.Tensor | None,
                          output: torch.Tensor) -> None:
        rows, columns = output.shape
        _check(library().fmm_reconstruct(self.rank, _dtype(output, products), products.data_ptr(), rows, columns,
                                         None if bias is None else bias.data_ptr(), output.data_ptr(),
                                         output.stride(0), _stream(products)),
               "fmm_reconstruct")
