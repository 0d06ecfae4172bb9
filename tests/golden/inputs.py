"""Seeded synthetic inputs shared by the golden-fixture generator, the tests,
``smoke()`` and ``bench.py``.

Inputs are drawn on the CPU with ``torch.Generator`` so the CPU oracle and the
GPU see identical bits: activations ~N(0, 1), weight ~N(0, 0.02) and
bias ~N(0, 0.02), all rounded to BF16 (the distributions of the benchmark
configurations; seeds A=0, W=1, bias=2 by default).
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch


def randn_bf16(shape, seed: int, std: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)


def randn_fp16(shape, seed: int, std: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(torch.float16)


def make_linear_inputs(M: int, K: int, N: int, seed: int = 0, bias: bool = False,
                       a_std: float = 1.0, w_std: float = 0.02):
    A = randn_bf16((M, K), seed, a_std)
    W = randn_bf16((N, K), seed + 1, w_std)
    b = randn_bf16((N,), seed + 2, w_std) if bias else None
    return A, W, b


def random_products(rank: int, bm: int, bn: int, seed: int) -> torch.Tensor:
    """FP16 stand-in for leaf products, used to pin the output transform alone."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn((rank, bm, bn), generator=g, dtype=torch.float32).to(torch.float16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def digest(array) -> str:
    if isinstance(array, torch.Tensor):
        array = array.contiguous().view(torch.int16).numpy() if array.element_size() == 2 \
            else array.contiguous().numpy()
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()
