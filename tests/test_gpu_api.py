"""Plan, operator and graph-rewrite behaviour on the GPU (mirrors the
reference's GPU tests, tests/test_rdna3.py:406-709 and
tests/test_inductor.py:114-203)."""

import pytest
import torch

from inputs import make_linear_inputs
from rdna3_fastmm import linear as linear_module
from rdna3_fastmm.linear import rdna3_linear, rdna3_rank7_linear, rdna3_rank48_linear
from rdna3_fastmm.runtime import LinearShapeFamily, Rank7Plan, Rank48Plan, Rank49Plan

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)
PLANS = [Rank7Plan, Rank48Plan, Rank49Plan]


def _plan(plan_type, *shape):
    return plan_type(*shape, DEVICE, dtype=torch.bfloat16, compute_dtype=torch.float16)


def _rel(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b))


@pytest.mark.parametrize("plan_type", PLANS)
def test_dynamic_and_packed_match_exact_small_product(plan_type):
    g = torch.Generator().manual_seed(11)
    x = torch.randint(-2, 3, (5, 6), generator=g).to(torch.bfloat16).to(DEVICE)
    w = torch.randint(-2, 3, (7, 6), generator=g).to(torch.bfloat16).to(DEVICE)
    expected = (x.float() @ w.float().T).to(torch.bfloat16)
    plan = _plan(plan_type, 5, 6, 7)
    ws = plan.allocate_workspace(max_free_memory_fraction=0.1)
    packed = plan.pack_weight(w, max_free_memory_fraction=0.1)
    pws = plan.allocate_workspace(max_free_memory_fraction=0.1, prepacked_right=True)
    for _ in range(3):
        assert torch.equal(plan.run_linear(x, w, ws), expected)
        assert torch.equal(plan.run_linear_packed(x, packed, pws), expected)
    snapshot = plan.run_linear_packed(x, packed, pws).clone()
    w.zero_()
    assert torch.equal(plan.run_linear_packed(x, packed, pws), snapshot)
    assert pws.right_transformed is None


@pytest.mark.parametrize("plan_type", PLANS)
def test_native_weight_layout_bias_and_bitwise_dynamic_equals_prepacked(plan_type):
    x, w, b = (t.to(DEVICE) for t in make_linear_inputs(257, 263, 269, seed=19, bias=True, w_std=1.0))
    reference = x.double() @ w.double().T + b.double()
    plan = _plan(plan_type, 257, 263, 269)
    dynamic = plan.run_linear(x, w, plan.allocate_workspace(0.1), b)
    packed = plan.pack_weight(w, 0.1)
    prepacked = plan.run_linear_packed(x, packed, plan.allocate_workspace(0.1, prepacked_right=True), b)
    assert torch.isfinite(dynamic).all()
    assert _rel(dynamic, reference) < 5e-3
    assert torch.equal(dynamic, prepacked)
    assert packed.source_shape == (269, 263)


def test_output_buffer_is_used_and_validated():
    x, w, _ = (t.to(DEVICE) if t is not None else None for t in make_linear_inputs(64, 64, 64))
    plan = _plan(Rank7Plan, 64, 64, 64)
    ws = plan.allocate_workspace(0.1)
    out = torch.empty((64, 64), device=DEVICE, dtype=torch.bfloat16)
    assert plan.run_linear(x, w, ws, output=out).data_ptr() == out.data_ptr()
    with pytest.raises(ValueError, match="overlap"):
        plan.run_linear(x, w, ws, output=x)
    with pytest.raises(ValueError, match="shape"):
        plan.run_linear(x[:32], w, ws)
    with pytest.raises(ValueError, match="contiguous"):
        plan.run_linear(x.t(), w, ws)
    with pytest.raises(ValueError, match="autograd"):
        plan.run_linear(x.clone().requires_grad_(True), w, ws)
    with pytest.raises(ValueError, match="dtype"):
        plan.run_linear(x.half(), w, ws)
    other = _plan(Rank49Plan, 64, 64, 64)
    with pytest.raises(ValueError, match="workspace does not match"):
        plan.run_linear(x, w, other.allocate_workspace(0.1))
    with pytest.raises(ValueError, match="dynamic workspace"):
        plan.run_linear(x, w, plan.allocate_workspace(0.1, prepacked_right=True))


def test_packed_weight_reuses_across_rows_and_rejects_other_shape():
    g = torch.Generator().manual_seed(37)
    w = torch.randn((7, 6), generator=g).to(torch.bfloat16).to(DEVICE)
    packed = _plan(Rank7Plan, 5, 6, 7).pack_weight(w, 0.1)
    x = torch.randn((9, 6), generator=g).to(torch.bfloat16).to(DEVICE)
    target = _plan(Rank7Plan, 9, 6, 7)
    assert torch.equal(target.run_linear(x, w, target.allocate_workspace(0.1)),
                       target.run_linear_packed(x, packed, target.allocate_workspace(0.1, prepacked_right=True)))
    other = _plan(Rank7Plan, 9, 8, 7)
    with pytest.raises(ValueError, match="packed Linear weight shape"):
        other.run_linear_packed(torch.zeros((9, 8), device=DEVICE, dtype=torch.bfloat16), packed,
                                other.allocate_workspace(0.1, prepacked_right=True))


@pytest.mark.parametrize("op", [rdna3_linear, rdna3_rank7_linear, rdna3_rank48_linear])
def test_linear_ops_support_leading_dimensions(op):
    g = torch.Generator().manual_seed(29)
    x = torch.randn((2, 17, 19), generator=g).to(torch.bfloat16).to(DEVICE)
    w = torch.randn((23, 19), generator=g).to(torch.bfloat16).to(DEVICE)
    b = torch.randn((23,), generator=g).to(torch.bfloat16).to(DEVICE)
    reference = x.double() @ w.double().T + b.double()
    out = op(x, w, b)
    assert out.shape == (2, 17, 23)
    assert _rel(out, reference) < 5e-3


class _FunctionalModel(torch.nn.Module):
    """Calls F.linear directly, so a symbolic trace records
    ``torch._C._nn.linear`` call_function nodes, as Dynamo graphs do."""

    def __init__(self, inner, columns, out):
        super().__init__()
        self.w1 = torch.nn.Parameter(torch.randn(columns, inner, dtype=torch.bfloat16) * 0.1,
                                     requires_grad=False)
        self.b1 = torch.nn.Parameter(torch.randn(columns, dtype=torch.bfloat16) * 0.1,
                                     requires_grad=False)
        self.w2 = torch.nn.Parameter(torch.randn(out, columns, dtype=torch.bfloat16) * 0.1,
                                     requires_grad=False)

    def forward(self, x):
        return torch.nn.functional.linear(torch.nn.functional.linear(x, self.w1, self.b1), self.w2)


def test_fx_rewrite_selects_an_admitted_shape(monkeypatch):
    monkeypatch.setattr(Rank7Plan, "linear_shape_families", (LinearShapeFamily(34, 34, 19, 23, True),))
    model = _FunctionalModel(19, 23, 11).to(DEVICE)
    x = torch.randn((2, 17, 19), device=DEVICE, dtype=torch.bfloat16)
    gm = torch.fx.symbolic_trace(model)
    with torch.no_grad():
        expected = model(x)
        rewritten = linear_module.rewrite_eligible_linears(gm, [x])
        targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
        assert rewritten == 1
        assert linear_module.RDNA3_RANK7_LINEAR_OP in targets
        assert _rel(gm(x), expected) < 1e-2


def test_fx_rewrite_leaves_unmeasured_shapes_on_cublas():
    model = _FunctionalModel(64, 64, 64).to(DEVICE)
    x = torch.randn((8, 64), device=DEVICE, dtype=torch.bfloat16)
    gm = torch.fx.symbolic_trace(model)
    with torch.no_grad():
        assert linear_module.rewrite_eligible_linears(gm, [x]) == 0


def test_compiled_model_runs_through_the_backend():
    # in-tree use: importing the backend module registers "rdna3-fastmm"
    # (an installed package registers it through its entry point)
    import rdna3_fastmm.inductor  # noqa: F401

    model = _FunctionalModel(64, 96, 32).to(DEVICE)
    x = torch.randn((4, 64), device=DEVICE, dtype=torch.bfloat16)
    with torch.no_grad():
        compiled = torch.compile(model, backend="rdna3-fastmm")
        assert _rel(compiled(x), model(x)) < 1e-2


def test_memory_guard_blocks_rewrite(monkeypatch):
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda device=None: (1024, 2**34))
    assert not linear_module._has_linear_memory_budget(Rank7Plan, (4096, 4096, 4096), DEVICE)


@pytest.mark.parametrize("plan_type", PLANS)
@pytest.mark.parametrize("prepacked", [False, True])
def test_linear_captures_into_a_cuda_graph(plan_type, prepacked):
    """After one eager call (which sets kernel attributes), a plan call is
    stream-ordered, synchronisation- and allocation-free, so it captures into a
    CUDA graph; replays give the eager bits for new inputs copied in place."""
    M, K, N = 520, 384, 776
    A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=True)
    A2 = make_linear_inputs(M, K, N, seed=5)[0]
    plan = _plan(plan_type, M, K, N)
    x, w, b = A.to(DEVICE), W.to(DEVICE), bias.to(DEVICE)
    out = torch.empty((M, N), device=DEVICE, dtype=torch.bfloat16)
    if prepacked:
        packed = plan.pack_weight(w, 0.5)
        ws = plan.allocate_workspace(0.5, prepacked_right=True)
        call = lambda: plan.run_linear_packed(x, packed, ws, b, out)  # noqa: E731
    else:
        ws = plan.allocate_workspace(0.5)
        call = lambda: plan.run_linear(x, w, ws, b, out)  # noqa: E731
    call()
    torch.cuda.synchronize()
    expected_first = out.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call()  # warm the side stream once, as torch.cuda.graph expects
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), expected_first.view(torch.int16))
    x.copy_(A2.to(DEVICE))
    graph.replay()
    torch.cuda.synchronize()
    eager = (plan.run_linear_packed(x, packed, ws, b) if prepacked else plan.run_linear(x, w, ws, b))
    assert torch.equal(out.view(torch.int16), eager.view(torch.int16))
