"""The C ABI library loads without a GPU, exports every symbol the header
declares, and answers its pure-host entry points."""

import ctypes
import re
from pathlib import Path

import pytest

from rdna3_fastmm import _native
from rdna3_fastmm.runtime import MatrixShape

HEADER = Path(__file__).resolve().parent.parent / "include" / "fmm_sm100.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(fmm_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_path():
    names = declared_functions()
    for required in ("fmm_transform_a", "fmm_transform_w", "fmm_leaf_gemm", "fmm_reconstruct",
                     "fmm_linear", "fmm_plan_dims", "fmm_last_error_string"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _native.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _native._SIGNATURES, f"{name} has no ctypes signature"


@pytest.mark.parametrize("scheme,s", [("rank7", 2), ("rank48", 4), ("rank49", 4)])
@pytest.mark.parametrize("shape", [(1, 1, 1), (5, 6, 7), (257, 263, 269), (8214, 12288, 4608), (65536, 4608, 12288)])
def test_plan_dims_match_matrix_shape(scheme, s, shape):
    d = _native.plan_dims(scheme, *shape)
    m = MatrixShape.from_dimensions(*shape, s)
    rank = {"rank7": 7, "rank48": 48, "rank49": 49}[scheme]
    assert (d.scheme_size, d.rank) == (s, rank)
    assert (d.bm, d.bk, d.bn) == (m.block_rows, m.block_inner, m.block_columns)
    assert (d.ldk, d.ldp) == (m.inner_pitch, m.column_pitch)
    assert d.ldk % 8 == 0 and d.ldp % 8 == 0
    assert d.left_elements == rank * m.block_rows * m.inner_pitch
    assert d.right_elements == rank * m.block_columns * m.inner_pitch
    assert d.product_elements == rank * m.block_rows * m.column_pitch


def test_host_side_errors_need_no_gpu():
    lib = _native.library()
    dims = _native.FmmDims()
    assert lib.fmm_plan_dims(5, 4, 4, 4, ctypes.byref(dims)) == _native.FMM_ERR_UNSUPPORTED
    assert "unknown scheme" in _native.last_error()
    assert lib.fmm_plan_dims(7, 0, 4, 4, ctypes.byref(dims)) == _native.FMM_ERR_INVALID_ARGUMENT
    assert lib.fmm_transform_a(7, 0, None, 4, 4, 4, None, None) == _native.FMM_ERR_INVALID_ARGUMENT
    fake_ptr = ctypes.c_void_p(0x1000)
    assert lib.fmm_transform_a(7, 5, fake_ptr, 4, 4, 4, fake_ptr, None) == _native.FMM_ERR_UNSUPPORTED
    assert lib.fmm_set_wait_timeout_ns(0) == _native.FMM_ERR_INVALID_ARGUMENT
    fake = ctypes.c_void_p(0x1000)
    rc = lib.fmm_linear_noalloc(7, fake, fake, None, fake, 8192, 8192, 8192, None)
    assert rc == _native.FMM_ERR_TOO_LARGE
    # rank 343 has no BF16 form: refused up front, naming the entry point
    rc = lib.fmm_linear_noalloc(343, fake, fake, None, fake, 64, 64, 64, None)
    assert rc == _native.FMM_ERR_UNSUPPORTED
    assert "fmm_linear_noalloc" in _native.last_error()
    # 32 MiB + 256 B of planes (rank 7, 166 x 2704 x 3184): refused before any launch
    rc = lib.fmm_linear_noalloc(7, fake, fake, None, fake, 166, 2704, 3184, None)
    assert rc == _native.FMM_ERR_TOO_LARGE
    with pytest.raises(ValueError, match="unknown scheme"):
        _native.check(lib.fmm_plan_dims(3, 4, 4, 4, ctypes.byref(dims)), "fmm_plan_dims")


def test_version():
    assert _native.library().fmm_version() >= 100


def test_rank343_plan_dims():
    d = _native.plan_dims("rank343", 16384, 16384, 16384)
    assert (d.scheme_size, d.rank, d.bm, d.bk, d.bn) == (8, 343, 2048, 2048, 2048)
    assert d.left_elements == 343 * 2048 * 2048
    m = MatrixShape.from_dimensions(67, 71, 73, 8)
    d = _native.plan_dims("rank343", 67, 71, 73)
    assert (d.bm, d.bk, d.bn, d.ldk, d.ldp) == (m.block_rows, m.block_inner, m.block_columns,
                                                m.inner_pitch, m.column_pitch)


def test_newer_entry_points_validate_on_the_host():
    lib = _native.library()
    fake = ctypes.c_void_p(0x1000)
    # paired transform: null operands, short leading dimension, misaligned planes
    assert lib.fmm_transform_aw(7, 0, None, 4, 4, 4, fake, fake, 4, 4, fake, None) == \
        _native.FMM_ERR_INVALID_ARGUMENT
    assert lib.fmm_transform_aw(7, 0, fake, 4, 8, 4, fake, fake, 4, 8, fake, None) == \
        _native.FMM_ERR_INVALID_ARGUMENT
    odd = ctypes.c_void_p(0x1002)
    assert lib.fmm_transform_aw(7, 0, fake, 4, 4, 4, odd, fake, 4, 4, fake, None) == \
        _native.FMM_ERR_MISALIGNED
    # gathering reconstruct: destination count and pointers
    dests = (ctypes.c_void_p * 9)(*([0x1000] * 9))
    for ndest in (0, 9):
        assert lib.fmm_reconstruct_gather(48, 0, fake, 8, 8, None, dests, ndest, 8, None) == \
            _native.FMM_ERR_INVALID_ARGUMENT
    assert "ndest" in _native.last_error()
    nulls = (ctypes.c_void_p * 2)(0x1000, None)
    assert lib.fmm_reconstruct_gather(48, 0, fake, 8, 8, None, nulls, 2, 8, None) == \
        _native.FMM_ERR_INVALID_ARGUMENT
    # rank 343 is FP16 only and has no gathering reconstruct
    assert lib.fmm_transform_a(343, 0, fake, 16, 16, 16, fake, None) == _native.FMM_ERR_UNSUPPORTED
    assert "FP16" in _native.last_error()
    # IPC: null arguments are refused before any driver call
    assert lib.fmm_ipc_export(None, None, None) == _native.FMM_ERR_INVALID_ARGUMENT
    assert lib.fmm_ipc_close(None) == _native.FMM_ERR_INVALID_ARGUMENT
