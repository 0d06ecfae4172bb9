"""torch.compile backend and external matmul without a GPU (mirrors the
reference's tests/test_inductor.py:21-111)."""

import torch

from rdna3_fastmm import external_mm, inductor, linear


def test_external_mm_falls_back_to_torch_mm_on_cpu():
    left = torch.randn(8, 6, dtype=torch.float16)
    right = torch.randn(6, 5, dtype=torch.float16)
    out = torch.empty(8, 5, dtype=torch.float16)
    with torch.no_grad():
        external_mm.rdna3_rank49_dynamic_v1_out(left, right, out=out)
    torch.testing.assert_close(out, torch.mm(left, right))


def test_compile_backend_passes_options_through_when_disabled(monkeypatch):
    captured = {}

    def fake_compile(gm, inputs, options):
        captured["options"] = options
        return "compiled"

    monkeypatch.setattr(torch._inductor, "compile", fake_compile)
    monkeypatch.setattr(inductor, "_enable_external_matmul", lambda: False)
    gm = torch.fx.symbolic_trace(torch.nn.Linear(4, 4))
    assert inductor.compile_backend(gm, [torch.randn(2, 4)], options={"foo": 1}) == "compiled"
    assert captured["options"]["foo"] == 1
    assert "external_matmul" not in captured["options"] or \
        external_mm.rdna3_rank49_dynamic_v1_out not in captured["options"]["external_matmul"]


def test_compile_backend_registers_external_matmul_when_enabled(monkeypatch):
    captured = {}
    monkeypatch.setattr(torch._inductor, "compile",
                        lambda gm, inputs, options: captured.setdefault("options", options))
    monkeypatch.setattr(inductor, "_enable_external_matmul", lambda: True)
    monkeypatch.setattr(inductor, "rewrite_eligible_linears", lambda gm, inputs: 0)
    gm = torch.fx.symbolic_trace(torch.nn.Linear(4, 4))
    inductor.compile_backend(gm, [torch.randn(2, 4)], mode=None, options={"external_matmul": []})
    options = captured["options"]
    assert external_mm.rdna3_rank49_dynamic_v1_out in options["external_matmul"]
    assert options["max_autotune_gemm"] is True
    assert options["triton.cudagraphs"] is False


def test_backend_is_registered_under_the_reference_name():
    from torch._dynamo import list_backends

    assert "rdna3-fastmm" in list_backends(exclude_tags=())


def test_operators_are_registered():
    for name in ("linear", "linear_rank7", "linear_rank48"):
        assert hasattr(torch.ops.rdna3_fastmm, name)


def test_cpu_linears_are_not_rewritten():
    model = torch.nn.Sequential(torch.nn.Linear(8, 8), torch.nn.ReLU()).to(torch.bfloat16)
    gm = torch.fx.symbolic_trace(model)
    assert linear.rewrite_eligible_linears(gm, [torch.randn(4, 8, dtype=torch.bfloat16)]) == 0


def test_pyproject_registers_named_dynamo_backend():
    import tomllib
    from pathlib import Path

    pyproject = tomllib.loads((Path(__file__).resolve().parent.parent / "pyproject.toml").read_text())
    assert pyproject["project"]["entry-points"]["torch_dynamo_backends"] == {
        "rdna3-fastmm": "rdna3_fastmm.inductor:compile_backend"
    }


def test_default_mode_resolves_to_default_options(monkeypatch):
    captured = {}
    monkeypatch.setattr(torch._inductor, "compile",
                        lambda gm, inputs, options: captured.__setitem__("options", options))
    monkeypatch.setattr(inductor, "_enable_external_matmul", lambda: False)
    gm = torch.fx.symbolic_trace(lambda v: v.cos())
    inductor.compile_backend(gm, [torch.randn(4)])
    assert captured["options"] == {}
    inductor.compile_backend(gm, [torch.randn(4)], mode="reduce-overhead")
    assert captured["options"] == {"triton.cudagraphs": True}


def test_external_mm_admitted_shape_on_cpu_falls_back(monkeypatch):
    """A shape in the plan's table still goes to torch.mm when the plan itself
    refuses the tensors (here: a CPU device)."""
    from rdna3_fastmm.runtime import Rank49Plan

    monkeypatch.setattr(Rank49Plan, "dynamic_shapes", frozenset({(8, 6, 5)}))
    left = torch.randn(8, 6, dtype=torch.float16)
    right = torch.randn(6, 5, dtype=torch.float16)
    out = torch.empty(8, 5, dtype=torch.float16)
    with torch.no_grad():
        assert not external_mm.is_rank49_dynamic_eligible(left, right, out)
        external_mm.rdna3_rank49_dynamic_v1_out(left, right, out=out)
    torch.testing.assert_close(out, torch.mm(left, right))
