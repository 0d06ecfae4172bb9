"""ctypes binding of ``libfmm_sm100.so`` (declared in ``include/fmm_sm100.h``).

The library is built in-tree (``rdna3-fastmm_b200/build.py``) into
``rdna3_fastmm/_lib``.  There is no fallback: when the library is missing, or
a call fails, the error is raised to the caller.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "_lib" / "libfmm_sm100.so"

FMM_OK = 0
FMM_ERR_INVALID_ARGUMENT = 1
FMM_ERR_MISALIGNED = 2
FMM_ERR_UNSUPPORTED = 3
FMM_ERR_CUDA = 4
FMM_ERR_DEVICE_TIMEOUT = 5
FMM_ERR_TOO_LARGE = 6
FMM_STATUS_TIMEOUT = 1
FMM_LINEAR_PREPACKED = 1
FMM_RIGHT_KN = 2
FMM_DTYPE_BF16 = 0
FMM_DTYPE_F16 = 1
FMM_DTYPE_BF16_BF16 = 2

SCHEME_IDS = {"rank7": 7, "rank48": 48, "rank49": 49, "rank343": 343}


class NativeLibraryError(RuntimeError):
    """The sm_100a library is missing, not loadable, or a call failed."""


class FmmDims(ctypes.Structure):
    _fields_ = [
        ("scheme_size", ctypes.c_int64),
        ("rank", ctypes.c_int64),
        ("bm", ctypes.c_int64),
        ("bk", ctypes.c_int64),
        ("bn", ctypes.c_int64),
        ("ldk", ctypes.c_int64),
        ("ldp", ctypes.c_int64),
        ("left_elements", ctypes.c_int64),
        ("right_elements", ctypes.c_int64),
        ("product_elements", ctypes.c_int64),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SIGNATURES = {
    "fmm_version": ([], ctypes.c_int),
    "fmm_last_error_string": ([], ctypes.c_char_p),
    "fmm_plan_dims": ([ctypes.c_int, _I64, _I64, _I64, ctypes.POINTER(FmmDims)], ctypes.c_int),
    "fmm_transform_a": ([ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _I64, _P, _P], ctypes.c_int),
    "fmm_transform_w": ([ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _I64, _P, _P], ctypes.c_int),
    "fmm_transform_b": ([ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _I64, _P, _P], ctypes.c_int),
    "fmm_leaf_gemm": ([ctypes.c_int, _P, _P, _I64, _I64, _I64, _P, _P], ctypes.c_int),
    "fmm_leaf_gemm_bf16": ([ctypes.c_int, _P, _P, _I64, _I64, _I64, _P, _P], ctypes.c_int),
    "fmm_ipc_export": ([_P, ctypes.POINTER(ctypes.c_ubyte), ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "fmm_ipc_import": (
        [ctypes.POINTER(ctypes.c_ubyte), ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p),
         ctypes.POINTER(ctypes.c_void_p)],
        ctypes.c_int,
    ),
    "fmm_ipc_close": ([_P], ctypes.c_int),
    "fmm_copy_async": ([_P, _P, ctypes.c_uint64, _P], ctypes.c_int),
    "fmm_transform_aw": (
        [ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _I64, _P, _P, _I64, _I64, _P, _P], ctypes.c_int,
    ),
    "fmm_reconstruct": ([ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _P, _P, _I64, _P], ctypes.c_int),
    "fmm_reconstruct_gather": (
        [ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _P, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
         _I64, _P],
        ctypes.c_int,
    ),
    "fmm_linear": (
        [ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, ctypes.c_uint, _P],
        ctypes.c_int,
    ),
    "fmm_linear_noalloc": ([ctypes.c_int, _P, _P, _P, _P, _I64, _I64, _I64, _P], ctypes.c_int),
    "fmm_set_sm_budget": ([ctypes.c_int], ctypes.c_int),
    "fmm_set_wait_timeout_ns": ([ctypes.c_uint64], ctypes.c_int),
    "fmm_device_status": (
        [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32), ctypes.c_int],
        ctypes.c_int,
    ),
    "fmm_test_bounded_wait": ([ctypes.c_uint64, _P], ctypes.c_int),
}


@lru_cache(maxsize=None)
def library() -> ctypes.CDLL:
    if not LIBRARY_PATH.exists():
        raise NativeLibraryError(
            f"{LIBRARY_PATH} is missing; build it with `python rdna3-fastmm_b200/build.py`"
        )
    try:
        lib = ctypes.CDLL(str(LIBRARY_PATH))
    except OSError as error:
        raise NativeLibraryError(f"cannot load {LIBRARY_PATH}: {error}") from error
    for name, (args, result) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = result
    return lib


def last_error() -> str:
    raw = library().fmm_last_error_string()
    return raw.decode() if raw else ""


def check(code: int, what: str) -> None:
    if code == FMM_OK:
        return
    message = f"{what}: {last_error()} (libfmm_sm100 error {code})"
    if code in (FMM_ERR_INVALID_ARGUMENT, FMM_ERR_MISALIGNED, FMM_ERR_UNSUPPORTED, FMM_ERR_TOO_LARGE):
        raise ValueError(message)
    raise NativeLibraryError(message)


def plan_dims(scheme: str, rows: int, inner: int, columns: int) -> FmmDims:
    dims = FmmDims()
    check(library().fmm_plan_dims(SCHEME_IDS[scheme], rows, inner, columns, ctypes.byref(dims)),
          "fmm_plan_dims")
    return dims


def _ptr(tensor) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def _stream(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def dtype_id(dtype, plane_dtype=None) -> int:
    """Precision id of a call: operand/output type ``dtype`` with planes of
    ``plane_dtype`` (FP16 when omitted)."""
    import torch

    plane_dtype = torch.float16 if plane_dtype is None else plane_dtype
    if dtype == torch.bfloat16 and plane_dtype == torch.float16:
        return FMM_DTYPE_BF16
    if dtype == torch.float16 and plane_dtype == torch.float16:
        return FMM_DTYPE_F16
    if dtype == torch.bfloat16 and plane_dtype == torch.bfloat16:
        return FMM_DTYPE_BF16_BF16
    raise ValueError(f"libfmm_sm100 takes BF16 or FP16 operands with FP16 planes, or BF16 operands "
                     f"with BF16 planes, not {dtype} with {plane_dtype} planes")


def transform_a(scheme: str, A, L) -> None:
    M, K = A.shape
    check(library().fmm_transform_a(SCHEME_IDS[scheme], dtype_id(A.dtype, L.dtype), _ptr(A), M, K, A.stride(0),
                                    _ptr(L), _stream(A.device)), "fmm_transform_a")


def transform_w(scheme: str, W, Rt) -> None:
    N, K = W.shape
    check(library().fmm_transform_w(SCHEME_IDS[scheme], dtype_id(W.dtype, Rt.dtype), _ptr(W), N, K, W.stride(0),
                                    _ptr(Rt), _stream(W.device)), "fmm_transform_w")


def transform_aw(scheme: str, A, L, W, Rt) -> None:
    """Both input-side transforms of a dynamic linear in one launch."""
    M, K = A.shape
    N = W.shape[0]
    check(library().fmm_transform_aw(SCHEME_IDS[scheme], dtype_id(A.dtype, L.dtype), _ptr(A), M, K, A.stride(0),
                                     _ptr(L), _ptr(W), N, W.stride(0), _ptr(Rt), _stream(A.device)),
          "fmm_transform_aw")


def transform_b(scheme: str, B, Rt) -> None:
    K, N = B.shape
    check(library().fmm_transform_b(SCHEME_IDS[scheme], dtype_id(B.dtype, Rt.dtype), _ptr(B), K, N, B.stride(0),
                                    _ptr(Rt), _stream(B.device)), "fmm_transform_b")


def leaf_gemm(rank: int, L, Rt, bm: int, bn: int, bk: int, P) -> None:
    """Leaf products on FP16 planes, or on BF16 planes when L is BF16."""
    import torch

    if L.dtype == torch.bfloat16:
        check(library().fmm_leaf_gemm_bf16(rank, _ptr(L), _ptr(Rt), bm, bn, bk, _ptr(P), _stream(L.device)),
              "fmm_leaf_gemm_bf16")
        return
    check(library().fmm_leaf_gemm(rank, _ptr(L), _ptr(Rt), bm, bn, bk, _ptr(P), _stream(L.device)),
          "fmm_leaf_gemm")


def reconstruct(scheme: str, P, M: int, N: int, bias, C) -> None:
    check(library().fmm_reconstruct(SCHEME_IDS[scheme], dtype_id(C.dtype, P.dtype), _ptr(P), M, N, _ptr(bias),
                                    _ptr(C), C.stride(0), _stream(P.device)), "fmm_reconstruct")


IPC_HANDLE_BYTES = 64


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(IPC handle bytes, offset) of the device allocation holding ``ptr``."""
    handle = (ctypes.c_ubyte * IPC_HANDLE_BYTES)()
    offset = ctypes.c_uint64()
    check(library().fmm_ipc_export(ptr, handle, ctypes.byref(offset)), "fmm_ipc_export")
    return bytes(handle), offset.value


def ipc_import(handle: bytes, offset: int) -> tuple[int, int]:
    """Map a peer's exported allocation: (mapping base, address at offset)."""
    raw = (ctypes.c_ubyte * IPC_HANDLE_BYTES).from_buffer_copy(handle)
    base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
    check(library().fmm_ipc_import(raw, offset, ctypes.byref(base), ctypes.byref(ptr)), "fmm_ipc_import")
    return int(base.value), int(ptr.value)


def ipc_close(base: int) -> None:
    check(library().fmm_ipc_close(base), "fmm_ipc_close")


def copy_async(dst: int, src: int, nbytes: int, stream: int) -> None:
    """Device-to-device copy (``dst`` may be a peer mapping) queued on ``stream``."""
    check(library().fmm_copy_async(dst, src, nbytes, stream), "fmm_copy_async")


def reconstruct_gather(scheme: str, P, M: int, N: int, bias, dests: list[int], ldc: int, dtype) -> None:
    """Output transform storing this rank's rows into every buffer in
    ``dests`` (device addresses of this rank's first row in the own and the
    peers' gathered outputs, leading dimension ``ldc``)."""
    array = (ctypes.c_void_p * len(dests))(*dests)
    check(library().fmm_reconstruct_gather(SCHEME_IDS[scheme], dtype_id(dtype, P.dtype), _ptr(P), M, N,
                                           _ptr(bias),
                                           array, len(dests), ldc, _stream(P.device)),
          "fmm_reconstruct_gather")


def linear(scheme: str, A, W, bias, C, L, Rt, P, prepacked: bool, right_kn: bool = False) -> None:
    """C = A @ W^T (+ bias); with ``right_kn`` W is a [K, N] right matrix and
    C = A @ W.  ``prepacked``: Rt already holds the right planes."""
    M, K = A.shape
    N = C.shape[1]
    flags = (FMM_LINEAR_PREPACKED if prepacked else 0) | (FMM_RIGHT_KN if right_kn else 0)
    check(library().fmm_linear(SCHEME_IDS[scheme], dtype_id(A.dtype, L.dtype), _ptr(A), _ptr(W), _ptr(bias),
                               _ptr(C), M, K, N, _ptr(L), _ptr(Rt), _ptr(P), flags, _stream(A.device)),
          "fmm_linear")


def linear_noalloc(scheme: str, A, W, bias, C) -> int:
    """Raw return code of fmm_linear_noalloc (callers decide how to react)."""
    M, K = A.shape
    N = C.shape[1]
    return library().fmm_linear_noalloc(SCHEME_IDS[scheme], _ptr(A), _ptr(W), _ptr(bias), _ptr(C),
                                        M, K, N, _stream(A.device))


def set_sm_budget(sms: int) -> None:
    """Cap the SMs one launch may fill (0 = all); see fmm_set_sm_budget."""
    check(library().fmm_set_sm_budget(sms), "fmm_set_sm_budget")


def set_wait_timeout_ns(timeout_ns: int) -> None:
    check(library().fmm_set_wait_timeout_ns(timeout_ns), "fmm_set_wait_timeout_ns")


def device_status(device_index: int, reset: bool = False) -> tuple[int, int]:
    status = ctypes.c_uint32(0)
    site = ctypes.c_uint32(0)
    check(library().fmm_device_status(device_index, ctypes.byref(status), ctypes.byref(site),
                                      int(reset)), "fmm_device_status")
    return status.value, site.value


def test_bounded_wait(timeout_ns: int, device) -> None:
    check(library().fmm_test_bounded_wait(timeout_ns, _stream(device)), "fmm_test_bounded_wait")
