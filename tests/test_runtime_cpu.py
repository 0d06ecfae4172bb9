"""Runtime gate, plan validation and workspace arithmetic without a GPU
(mirrors the reference's CPU-safe tests in tests/test_rdna3.py:32-388, with
the GPU faked by monkeypatching as the reference does)."""

from types import SimpleNamespace

import pytest
import torch

from rdna3_fastmm import runtime
from rdna3_fastmm.runtime import (LinearShapeFamily, MatrixShape, Rank7Plan, Rank48Plan, Rank49Plan,
                                  unsupported_runtime_reason)


def configure_supported_runtime(monkeypatch):
    monkeypatch.setattr(torch.version, "cuda", "12.8")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda device: SimpleNamespace(major=10, minor=0, multi_processor_count=148))
    monkeypatch.setattr(torch, "__version__", "2.11.0+cu128")


def test_runtime_support_reason_accepts_tested_stack(monkeypatch):
    configure_supported_runtime(monkeypatch)
    assert unsupported_runtime_reason() is None


def test_runtime_support_reason_requires_cuda_build(monkeypatch):
    monkeypatch.setattr(torch.version, "cuda", None)
    assert unsupported_runtime_reason() == "requires a CUDA PyTorch build"


def test_runtime_support_reason_requires_available_gpu(monkeypatch):
    configure_supported_runtime(monkeypatch)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    assert unsupported_runtime_reason() == "requires an available CUDA GPU"


def test_runtime_support_reason_rejects_cpu_device(monkeypatch):
    configure_supported_runtime(monkeypatch)
    assert unsupported_runtime_reason(torch.device("cpu")) == "requires a CUDA GPU device"


def test_runtime_support_reason_describes_wrong_gpu(monkeypatch):
    configure_supported_runtime(monkeypatch)
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda device: SimpleNamespace(major=9, minor=0, multi_processor_count=132))
    assert unsupported_runtime_reason() == "tested only on sm_100 with 148 SMs; found sm_90 with 132"


@pytest.mark.parametrize("component,version,expected", [
    ("torch", "2.9.1+cu128", "tested only with PyTorch 2.11; found 2.9.1+cu128"),
    ("cuda", "13.0", "tested only with CUDA 12; found 13.0"),
])
def test_runtime_support_reason_describes_version_mismatch(monkeypatch, component, version, expected):
    configure_supported_runtime(monkeypatch)
    if component == "torch":
        monkeypatch.setattr(torch, "__version__", version)
    else:
        monkeypatch.setattr(torch.version, "cuda", version)
    assert unsupported_runtime_reason() == expected


def test_rank_49_shape_uses_padded_quarters():
    shape = MatrixShape.from_dimensions(257, 263, 269, 4)
    assert shape.dimensions == (257, 263, 269)
    assert (shape.block_rows, shape.block_inner, shape.block_columns) == (65, 66, 68)
    assert shape.workspace_elements(49) == 49 * (65 * 66 + 66 * 68 + 65 * 68)
    assert (shape.inner_pitch, shape.column_pitch) == (72, 72)


def test_shape_rejects_nonpositive_dimensions():
    with pytest.raises(ValueError, match="positive"):
        MatrixShape.from_dimensions(4, 0, 4, 4)


@pytest.mark.parametrize("plan", [Rank7Plan, Rank48Plan, Rank49Plan])
def test_plan_rejects_cpu_device(plan):
    with pytest.raises(ValueError, match="CUDA sm_100"):
        plan(4, 4, 4, torch.device("cpu"))


@pytest.mark.parametrize("plan", [Rank7Plan, Rank48Plan])
def test_plan_rejects_unsupported_precision(monkeypatch, plan):
    configure_supported_runtime(monkeypatch)
    with pytest.raises(ValueError, match="does not support"):
        plan(4, 4, 4, torch.device("cuda", 0), dtype=torch.bfloat16, compute_dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="does not support"):
        plan(4, 4, 4, torch.device("cuda", 0), dtype=torch.float32)


def test_precision_pairs_follow_the_reference(monkeypatch):
    """FP16 plans exist for rank 7 and rank 49 (reference runtime.py:785-790,
    852-858); rank 48 is BF16-in only (:828); only rank 49 has BF16 planes
    (:855), and a BF16 rank-49 plan without compute_dtype resolves to them."""
    configure_supported_runtime(monkeypatch)
    dev = torch.device("cuda", 0)
    for plan in (Rank7Plan, Rank49Plan):
        p = plan(4, 4, 4, dev)  # default dtype FP16
        assert (p.dtype, p.compute_dtype) == (torch.float16, torch.float16)
    with pytest.raises(ValueError, match="does not support"):
        Rank48Plan(4, 4, 4, dev)
    p = Rank49Plan(4, 4, 4, dev, dtype=torch.bfloat16)
    assert (p.dtype, p.compute_dtype) == (torch.bfloat16, torch.bfloat16)
    assert p.packed_weight_bytes == Rank49Plan(4, 4, 4, dev, dtype=torch.bfloat16,
                                               compute_dtype=torch.float16).packed_weight_bytes
    assert not p.is_linear_recommended(has_bias=False)
    with pytest.raises(ValueError, match="does not support"):
        Rank49Plan(4, 4, 4, dev, dtype=torch.float32)
    assert Rank49Plan.precision_pairs == frozenset({(torch.float16, torch.float16),
                                                    (torch.bfloat16, torch.bfloat16),
                                                    (torch.bfloat16, torch.float16)})


def test_mm_tables_hold_only_measured_b200_wins():
    for plan in (Rank7Plan, Rank48Plan, Rank49Plan):
        assert plan.dynamic_shapes == frozenset() and plan.prepacked_shapes == frozenset()


@pytest.mark.parametrize("plan,rank,s", [(Rank7Plan, 7, 2), (Rank48Plan, 48, 4), (Rank49Plan, 49, 4)])
def test_workspace_byte_formulas(monkeypatch, plan, rank, s):
    configure_supported_runtime(monkeypatch)
    p = plan(257, 263, 269, torch.device("cuda", 0), dtype=torch.bfloat16, compute_dtype=torch.float16)
    m = MatrixShape.from_dimensions(257, 263, 269, s)
    left = rank * m.block_rows * m.inner_pitch * 2
    right = rank * m.block_columns * m.inner_pitch * 2
    products = rank * m.block_rows * m.column_pitch * 2
    assert p.workspace_bytes == left + right + products
    assert p.prepacked_workspace_bytes == left + products
    assert p.packed_weight_bytes == p.packed_right_bytes == right


def test_byte_formulas_equal_the_reference_when_blocks_are_aligned(monkeypatch):
    configure_supported_runtime(monkeypatch)
    p = Rank48Plan(8192, 8192, 8192, torch.device("cuda", 0), dtype=torch.bfloat16,
                   compute_dtype=torch.float16)
    assert p.workspace_bytes == p.shape.workspace_elements(48) * 2


def test_memory_budget_raises_memory_error(monkeypatch):
    configure_supported_runtime(monkeypatch)
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda device=None: (1024, 2**34))
    p = Rank7Plan(1024, 1024, 1024, torch.device("cuda", 0), dtype=torch.bfloat16,
                  compute_dtype=torch.float16)
    with pytest.raises(MemoryError, match="budget"):
        p.allocate_workspace()
    with pytest.raises(ValueError, match="interval"):
        p.allocate_workspace(max_free_memory_fraction=1.5)


def test_dispatch_tables_hold_only_measured_b200_wins():
    """Measured on B200 against cuBLAS BF16: no configuration wins, so every
    family table is empty and nothing is routed to the reduced-rank path."""
    for plan in (Rank7Plan, Rank48Plan, Rank49Plan):
        for shape in [(4096, 4096, 12288), (4992, 16384, 4096), (8214, 12288, 4608), (8192, 8192, 8192)]:
            for bias in (False, True):
                assert not plan.has_measured_linear_win(shape, has_bias=bias, prepacked_weight=True)


def test_shape_family_matches_like_the_reference():
    family = LinearShapeFamily(3600, 4096, 4096, 12288, False)
    assert family.matches((4096, 4096, 12288), False)
    assert family.matches((3600, 4096, 12288), False)
    assert not family.matches((3599, 4096, 12288), False)
    assert not family.matches((4096, 4096, 12288), True)


def test_prepacked_families_extend_dynamic_ones(monkeypatch):
    monkeypatch.setattr(Rank7Plan, "linear_shape_families", (LinearShapeFamily(1, 10, 8, 8, False),))
    monkeypatch.setattr(Rank7Plan, "prepacked_linear_shape_families", (LinearShapeFamily(720, 720, 8, 8, True),))
    assert Rank7Plan.has_measured_linear_win((5, 8, 8), has_bias=False)
    assert not Rank7Plan.has_measured_linear_win((720, 8, 8), has_bias=True)
    assert Rank7Plan.has_measured_linear_win((720, 8, 8), has_bias=True, prepacked_weight=True)


def test_storage_overlap_detection():
    base = torch.empty(100)
    assert runtime._overlaps(base[:50], base[49:])
    assert not runtime._overlaps(base[:50], base[50:])
