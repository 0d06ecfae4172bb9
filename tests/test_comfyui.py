"""ComfyUI node (mirrors the reference's ``tests/test_comfyui.py``): node
contract, clone semantics, compile configuration, guard filter, runtime
rejection, registry metadata and the custom-node entry point -- all on CPU."""

import os
import subprocess
import sys
import tomllib
from pathlib import Path

import pytest

from rdna3_fastmm import comfyui

ROOT = Path(__file__).resolve().parents[1]
NODE_DIR = ROOT / "rdna3-fastmm_b200"


class FakeGuardEntry:
    def __init__(self, name):
        self.name = name


class FakeModel:
    def __init__(self):
        self.clone_arguments = []

    def clone(self, disable_dynamic=False):
        self.clone_arguments.append(disable_dynamic)
        return type(self)()


def test_guard_filter_skips_only_comfy_transformer_options():
    entries = [FakeGuardEntry("model.model_options['transformer_options']"),
               FakeGuardEntry("model.model_options['other']"), FakeGuardEntry("input_tensor")]
    assert comfyui.skip_comfy_transformer_option_guards(entries) == [False, True, True]


def test_compile_node_clones_and_wraps_only_diffusion_model(monkeypatch):
    captured = {}
    source = FakeModel()

    def backend(*args, **kwargs):
        return object()

    def set_compile_wrapper(*, model, backend, options, dynamic, keys):
        captured.update(model=model, backend=backend, options=options, dynamic=dynamic, keys=keys)

    monkeypatch.setattr(comfyui, "_unsupported_reason", lambda: None)
    monkeypatch.setattr(comfyui, "_load_compile_backend", lambda: backend)
    monkeypatch.setattr(comfyui, "_load_compile_setter", lambda: set_compile_wrapper)
    (compiled,) = comfyui.RDNA3FastMMCompile().compile_model(source)
    assert compiled is captured["model"] and compiled is not source
    assert source.clone_arguments == [True]
    assert captured["backend"] is backend
    assert captured["keys"] == ["diffusion_model"]
    assert captured["options"] == {"guard_filter_fn": comfyui.skip_comfy_transformer_option_guards}
    assert captured["dynamic"] is False


def test_compile_node_rejects_unsupported_runtime_before_cloning(monkeypatch):
    source = FakeModel()
    monkeypatch.setattr(comfyui, "_unsupported_reason", lambda: "unsupported test runtime")
    with pytest.raises(RuntimeError, match="Cannot enable RDNA3 FastMM: unsupported test runtime"):
        comfyui.RDNA3FastMMCompile().compile_model(source)
    assert source.clone_arguments == []


def test_compile_setter_requires_current_comfyui(monkeypatch):
    def missing(name):
        raise ModuleNotFoundError(f"No module named {name!r}", name=name)

    monkeypatch.setattr(comfyui, "import_module", missing)
    with pytest.raises(RuntimeError, match="RDNA3 FastMM requires ComfyUI 0.19.0 or newer"):
        comfyui._load_compile_setter()


def test_compile_setter_reraises_other_missing_modules(monkeypatch):
    def missing(name):
        raise ModuleNotFoundError("No module named 'numpy'", name="numpy")

    monkeypatch.setattr(comfyui, "import_module", missing)
    with pytest.raises(ModuleNotFoundError):
        comfyui._load_compile_setter()


@pytest.mark.parametrize("version", ((3, 11, 9), (3, 14, 0)))
def test_adapter_rejects_unsupported_python_before_importing_runtime(monkeypatch, version):
    monkeypatch.setattr(sys, "version_info", version)
    monkeypatch.setattr(comfyui, "import_module",
                        lambda name: pytest.fail("runtime must not load on unsupported Python"))
    assert comfyui._unsupported_reason() == "RDNA3 FastMM compilation requires Python 3.12 or 3.13"


def test_backend_loader_returns_the_compile_backend():
    from rdna3_fastmm.inductor import compile_backend

    assert comfyui._load_compile_backend() is compile_backend


def test_comfyui_node_contract_is_exported():
    node = comfyui.RDNA3FastMMCompile
    assert node.INPUT_TYPES() == {"required": {"model": ("MODEL",)}}
    assert node.RETURN_TYPES == ("MODEL",)
    assert node.FUNCTION == "compile_model"
    assert node.EXPERIMENTAL is True
    assert comfyui.NODE_CLASS_MAPPINGS == {"RDNA3FastMMCompile": node}
    assert comfyui.NODE_DISPLAY_NAME_MAPPINGS == {"RDNA3FastMMCompile": "RDNA3 FastMM Compile"}


def test_comfyui_registry_metadata_matches_node_requirements():
    pyproject = tomllib.loads((ROOT / "pyproject.toml").read_text())
    assert pyproject["tool"]["comfy"]["requires-comfyui"] == ">=0.19.0"
    assert pyproject["project"]["entry-points"]["torch_dynamo_backends"] == {
        "rdna3-fastmm": "rdna3_fastmm.inductor:compile_backend"}


def test_comfyui_archive_keeps_runtime():
    ignored = set((NODE_DIR / ".comfyignore").read_text().splitlines())
    assert "benchmarks/" in ignored
    assert {"rdna3_fastmm/", "csrc/", "__init__.py"}.isdisjoint(ignored)


def _run(script, tmp_path):
    stale = tmp_path / "rdna3_fastmm"
    stale.mkdir()
    (stale / "__init__.py").write_text("SOURCE = 'stale install'\n")
    env = {**os.environ, "PYTHONPATH": str(tmp_path)}
    subprocess.run([sys.executable, "-c", script], cwd=tmp_path, env=env, check=True, timeout=300)


LOADER = f"""
import importlib.util
import sys
spec = importlib.util.spec_from_file_location(
    "fastmm_custom_node", {str(NODE_DIR / "__init__.py")!r},
    submodule_search_locations=[{str(NODE_DIR)!r}])
module = importlib.util.module_from_spec(spec)
sys.modules["fastmm_custom_node"] = module
"""


def test_custom_node_entrypoint_loads_source_package(tmp_path):
    _run(LOADER + f"""
spec.loader.exec_module(module)
node = module.NODE_CLASS_MAPPINGS["RDNA3FastMMCompile"]
assert node.__module__ == "rdna3_fastmm.comfyui"
assert {str(NODE_DIR)!r} in sys.modules["rdna3_fastmm"].__file__
assert {str(NODE_DIR)!r} not in sys.path
""", tmp_path)


def test_custom_node_entrypoint_rejects_preloaded_conflict(tmp_path):
    _run("import rdna3_fastmm\n" + LOADER + """
try:
    spec.loader.exec_module(module)
except RuntimeError as error:
    assert "different rdna3_fastmm package is already loaded" in str(error)
else:
    raise AssertionError("preloaded conflicting package was accepted")
""", tmp_path)
