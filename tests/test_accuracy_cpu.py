"""Host-side checks of the error-gate helper (``rdna3_fastmm.accuracy``) on CPU
tensors: tile placement as the reference's harness places it, and the gate's
arithmetic on outputs whose errors are known."""

import math

import pytest
import torch

from inputs import make_linear_inputs
from rdna3_fastmm.accuracy import centred_tile_starts, error_gate


def test_tile_starts_are_centred_in_every_block():
    # 8214 rows in 4 blocks of 2054 (last 2052): tiles centred in each
    assert centred_tile_starts(8214, 16, 4) == [1019, 3073, 5127, 7180]
    assert centred_tile_starts(4096, 64, 2) == [992, 3040]
    with pytest.raises(ValueError):
        centred_tile_starts(100, 64, 4)


def test_gate_on_known_errors():
    M, K, N = 256, 96, 128
    A, W, bias = make_linear_inputs(M, K, N, seed=3, bias=True)
    exact = (A.double() @ W.double().T + bias.double())
    native = torch.nn.functional.linear(A.float(), W.float(), bias.float()).to(torch.bfloat16)

    same = error_gate(A, W, bias, native, 2, tile=32, native=native)
    assert same["ratio"] == pytest.approx(1.0)
    assert same["passes"] and same["nonfinite_outputs"] == 0
    assert same["samples"] == 4 * 32 * 32

    # an output rounded to BF16 from the exact product is at least as good as native
    rounded = exact.to(torch.bfloat16)
    better = error_gate(A, W, bias, rounded, 2, tile=32, native=native)
    assert better["ratio"] <= 1.0 + 1e-9

    # twice the native error everywhere fails the gate
    worse = (exact + 2.0 * (native.double() - exact)).to(torch.float64)
    failing = error_gate(A, W, bias, worse, 2, tile=32, native=native)
    assert failing["ratio"] == pytest.approx(2.0, rel=1e-6) and not failing["passes"]

    # a non-finite value outside the sampled tiles still fails it
    poisoned = native.clone()
    poisoned[0, 0] = float("nan")
    result = error_gate(A, W, bias, poisoned, 2, tile=32, native=native)
    assert result["nonfinite_outputs"] == 1 and not result["passes"]
    assert math.isfinite(result["rel_l2_vs_fp64"])
