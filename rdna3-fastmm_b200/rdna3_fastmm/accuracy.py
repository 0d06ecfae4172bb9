"""Error gate of the reduced-rank linear against an FP64 product.

The reference judges a candidate output by its relative L2 error on sampled
tiles against a high-precision product, divided by the error of the native
BF16 ``F.linear`` on the same samples (``benchmarks/benchmark.py:160-265`` of
chelokot/rdna3-fastmm: one centred ``tile x tile`` sample inside every
``s x s`` output macroblock, so every block row and block column of the
scheme is covered).  This module applies that protocol on the device with an
FP64 reference (FP64 products of the BF16 inputs, FP64 accumulation), and
counts non-finite values over the whole output, not only the samples.

The gate passes when the candidate's error is at most ``limit`` (1.2) times
the native error and no output is non-finite.
"""

from __future__ import annotations

import math

import torch

__all__ = ["centred_tile_starts", "error_gate", "GATE_LIMIT"]

GATE_LIMIT = 1.2


def centred_tile_starts(dimension: int, tile: int, scheme_size: int) -> list[int]:
    """First index of a centred ``tile`` inside each of the ``scheme_size``
    blocks of ``ceil(dimension / scheme_size)`` (the last block may be
    shorter)."""
    block = -(-dimension // scheme_size)
    starts = []
    for b in range(scheme_size):
        lo, hi = b * block, min((b + 1) * block, dimension)
        if hi - lo < tile:
            raise ValueError(f"block {b} of {dimension} holds fewer than {tile} positions")
        starts.append(lo + (hi - lo - tile) // 2)
    return starts


def _nonfinite(tensor: torch.Tensor, chunk_rows: int = 4096) -> int:
    count = 0
    for start in range(0, tensor.shape[0], chunk_rows):
        count += int((~torch.isfinite(tensor[start:start + chunk_rows])).sum())
    return count


@torch.no_grad()
def error_gate(A: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
               candidate: torch.Tensor, scheme_size: int, *, tile: int = 64,
               native: torch.Tensor | None = None, limit: float = GATE_LIMIT) -> dict:
    """Relative L2 error of ``candidate`` (``[M, N]``) and of native BF16
    against ``A @ weight^T (+ bias)`` in FP64 on the centred macroblock tiles.

    ``A`` may live on the CPU (a sharded job's full input); the sampled rows
    are moved to ``candidate``'s device.  ``native`` defaults to
    ``F.linear(A, weight, bias)`` computed on that device (it must then fit).
    """
    device = candidate.device
    M, N = candidate.shape
    if native is None:
        native = torch.nn.functional.linear(A.to(device), weight.to(device),
                                            None if bias is None else bias.to(device))
    row_starts = centred_tile_starts(M, tile, scheme_size)
    col_starts = centred_tile_starts(N, tile, scheme_size)
    w64 = weight.to(device).double()
    b64 = None if bias is None else bias.to(device).double()
    sq_ref = sq_cand = sq_native = 0.0
    for r in row_starts:
        a64 = A[r:r + tile].to(device).double()
        for c in col_starts:
            exact = a64 @ w64[c:c + tile].T
            if b64 is not None:
                exact += b64[c:c + tile]
            cand = candidate[r:r + tile, c:c + tile].double()
            nat = native[r:r + tile, c:c + tile].double()
            sq_ref += float(exact.square().sum())
            sq_cand += float(torch.where(torch.isfinite(cand), cand - exact, 0.0).square().sum())
            sq_native += float((nat - exact).square().sum())
    rel = math.sqrt(sq_cand / sq_ref)
    rel_native = math.sqrt(sq_native / sq_ref)
    nonfinite = _nonfinite(candidate)
    ratio = rel / rel_native if rel_native else None
    return {
        "rel_l2_vs_fp64": rel,
        "native_bf16_rel_l2": rel_native,
        "ratio": ratio,
        "limit": limit,
        "passes": ratio is not None and ratio <= limit and nonfinite == 0,
        "nonfinite_outputs": nonfinite,
        "samples": len(row_starts) * len(col_starts) * tile * tile,
        "tile": tile,
        "reference": "fp64 product of the BF16 inputs, centred tile per output macroblock",
    }
