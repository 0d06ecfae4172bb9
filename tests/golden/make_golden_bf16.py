"""Golden fixtures for BF16 planes, made by running the REFERENCE's own kernels.

The reference's ``Rank49Plan`` accepts the ``(bfloat16, bfloat16)`` precision
pair (``src/rdna3_fastmm/runtime.py:852-858``): BF16 inputs, BF16 transform
planes and BF16 leaf products.  Its generated rank-49 Triton kernels
(``src/rdna3_fastmm/generated/rank49_4x4x4.py``) are run here on CPU tensors
under ``TRITON_INTERPRET=1``, once, in a container that has the reference
checked out (``--reference``; never read at test time):

    python tests/golden/make_golden_bf16.py --reference <path-to-reference>

The interpreter truncates FP32 -> BF16 on store, so every kernel stores into
an FP32 buffer -- the exact FP32 value the kernel computed for each plane or
output element -- and the BF16 round-to-nearest-even a GPU store performs is
done by ``Tensor.to(torch.bfloat16)``.

Writes ``golden_bf16.json`` (SHA-256 digests) and ``golden_bf16.npz`` (the
full arrays of the small cases, as int16 bit patterns).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from inputs import digest, make_linear_inputs  # noqa: E402

SHAPES = [(5, 6, 7), (17, 19, 23), (257, 263, 269)]
SMALL = {(5, 6, 7), (17, 19, 23)}


def bf16_products(rank: int, bm: int, bn: int, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randn((rank, bm, bn), generator=g, dtype=torch.float32).to(torch.bfloat16)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference / "src"))
    import numpy as np
    import torch
    import triton
    from rdna3_fastmm.generated import rank49_4x4x4 as module

    s, rank = 4, 49
    record: dict = {"generator": "reference generated Triton kernels (rank 49, BF16 planes), "
                                 "TRITON_INTERPRET=1, FP32 stores rounded to BF16 by torch",
                    "triton": triton.__version__, "torch": torch.__version__, "cases": []}
    arrays: dict = {}
    for M, K, N in SHAPES:
        bm, bk, bn = -(-M // s), -(-K // s), -(-N // s)
        A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=True)
        L32 = torch.empty((rank, bm, bk), dtype=torch.float32)
        module.left_transform_kernel[(triton.cdiv(bm * bk, 256),)](A, L32, M, K, bm, bk, bm, bk, 256)
        R32 = torch.empty((rank, bk, bn), dtype=torch.float32)
        module.right_transform_weight_kernel[(triton.cdiv(bk, 4), triton.cdiv(bn, 64))](
            W, R32, N, K, bk, bn, 4, 64)
        L, Rw = L32.to(torch.bfloat16), R32.to(torch.bfloat16)
        P = bf16_products(rank, bm, bn, seed=3)
        outputs = {}
        for with_bias in (False, True):
            C32 = torch.zeros((M, N), dtype=torch.float32)
            grid = (triton.cdiv(bm * bn, 256),)
            if with_bias:
                module.output_transform_bias_kernel[grid](P, C32, bias, bm, bn, M, N, bm, bn, 256)
            else:
                module.output_transform_kernel[grid](P, C32, bm, bn, M, N, bm, bn, 256)
            outputs[with_bias] = C32.to(torch.bfloat16)
        record["cases"].append({
            "scheme": "rank49", "planes": "bf16", "shape": [M, K, N], "seed": 0, "product_seed": 3,
            "inputs": {"A": digest(A), "W": digest(W), "bias": digest(bias), "P": digest(P)},
            "left": digest(L), "weight": digest(Rw),
            "output": digest(outputs[False]), "output_bias": digest(outputs[True])})
        if (M, K, N) in SMALL:
            key = f"rank49_{M}x{K}x{N}"
            arrays[key + "_left"] = L.view(torch.int16).numpy()
            arrays[key + "_weight"] = Rw.view(torch.int16).numpy()
            arrays[key + "_output"] = outputs[False].view(torch.int16).numpy()
            arrays[key + "_output_bias"] = outputs[True].view(torch.int16).numpy()
        print("rank49 bf16", (M, K, N), "done", flush=True)
    (HERE / "golden_bf16.json").write_text(json.dumps(record, indent=1) + "\n")
    np.savez_compressed(HERE / "golden_bf16.npz", **arrays)


if __name__ == "__main__":
    main()
