"""The reference-side ctypes binding (``rdna3-fastmm_b200/examples/reference_binding.py``)
declares every entry point it calls with exactly the parameters
``include/fmm_sm100.h`` gives it, and binds the built library on a host
without a GPU."""

import ctypes
import importlib.util
import re
from pathlib import Path

import pytest

from rdna3_fastmm import _native

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "fmm_sm100.h"
BINDING = ROOT / "rdna3-fastmm_b200" / "examples" / "reference_binding.py"

C_TYPES = {
    "int": ctypes.c_int, "unsigned int": ctypes.c_uint, "int64_t": ctypes.c_int64,
    "uint64_t": ctypes.c_uint64, "fmm_stream_t": ctypes.c_void_p,
}


def load_binding():
    spec = importlib.util.spec_from_file_location("reference_binding", BINDING)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def header_parameters(name: str) -> list[str]:
    """Parameter types of ``name`` as the header declares them."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    match = re.search(rf"\b{name}\s*\(([^)]*)\)\s*;", text)
    assert match, name
    params = [p.strip() for p in match.group(1).split(",")]
    if params == ["void"]:
        return []
    return [re.sub(r"\s*\b\w+$", "", p) if not p.endswith("*") else p for p in params]


def ctype_of(c_param: str):
    if "*" in c_param:
        base = c_param.replace("const", "").replace("*", "").strip()
        return ("pointer", base)
    return C_TYPES[c_param.strip()]


def binding_type(t):
    if t is ctypes.c_void_p:
        return "void_ptr"
    if isinstance(t, type) and issubclass(t, ctypes._Pointer):
        return ("pointer", t._type_.__name__)
    return t


@pytest.mark.parametrize("name", sorted(load_binding().ARGTYPES))
def test_binding_matches_header(name):
    declared = header_parameters(name)
    bound = load_binding().ARGTYPES[name]
    assert len(bound) == len(declared), (name, declared)
    for c_param, t in zip(declared, bound):
        expected = ctype_of(c_param)
        got = binding_type(t)
        if isinstance(expected, tuple):
            if expected[1] in ("void", "unsigned char"):
                assert got == "void_ptr" or got[0] == "pointer", (name, c_param, t)
            else:  # a struct pointer: the struct's name
                assert got == ("pointer", "FmmDims") and expected[1] == "fmm_dims", (name, c_param, t)
        elif expected is ctypes.c_void_p:
            assert got == "void_ptr", (name, c_param, t)
        else:
            assert t is expected, (name, c_param, t)


@pytest.mark.parametrize("name", sorted(load_binding().ARGTYPES))
def test_binding_agrees_with_the_package_binding(name):
    """The package's own ctypes table and the reference-side stub give the
    same argument count for every shared entry point."""
    assert len(load_binding().ARGTYPES[name]) == len(_native._SIGNATURES[name][0])


def test_binding_loads_the_library_and_answers_host_calls():
    module = load_binding()
    lib = module.load(str(_native.LIBRARY_PATH))
    dims = module.FmmDims()
    assert lib.fmm_plan_dims(49, 8214, 12288, 4608, ctypes.byref(dims)) == module.FMM_OK
    assert (dims.bm, dims.bk, dims.bn, dims.ldk, dims.ldp) == (2054, 3072, 1152, 3072, 1152)
    # a null source is refused before anything touches a device
    assert lib.fmm_transform_a(7, module.FMM_DTYPE_BF16, None, 4, 4, 4, None, None) != module.FMM_OK
    assert b"null" in lib.fmm_last_error_string()
