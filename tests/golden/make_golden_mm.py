"""Golden fixtures for the FP16 plain-mm path, made by running the REFERENCE's
own kernels.

Run once in a container that has chelokot/rdna3-fastmm checked out (the path
is given by ``--reference``; it is never read at test time):

    python tests/golden/make_golden_mm.py --reference <path-to-reference>

The reference's generated Triton kernels for the schemes its FP16 plans admit
(rank 7 and rank 49: ``src/rdna3_fastmm/generated/rank{7_2x2x2,49_4x4x4}.py``)
run on CPU tensors under ``TRITON_INTERPRET=1`` with FP16 operands, as
``Rank7Plan.run`` / ``Rank49Plan.run`` launch them (``runtime.py:597-698``):
``left_transform_kernel`` on ``A[M, K]``, ``right_transform_kernel`` on the
contiguous ``B[K, N]`` and ``output_transform_kernel`` into an FP16 ``C``
(FP32 -> FP16 stores are correctly rounded in the interpreter); and, for the
FP16 linear plans, ``right_transform_weight_kernel`` on the native
``weight[N, K] = B^T`` and ``output_transform_bias_kernel`` with an FP16 bias.

Writes ``golden_mm.json`` (SHA-256 digests) and ``golden_mm.npz`` (full
arrays of the small cases).
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

from inputs import digest, randn_fp16, random_products  # noqa: E402

CASES = {
    "rank7": [(5, 6, 7), (17, 19, 23), (257, 263, 269)],
    "rank49": [(5, 6, 7), (17, 19, 23), (257, 263, 269)],
}
SMALL = {(5, 6, 7), (17, 19, 23)}
BLOCK_ELEMENTS = 256


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference / "src"))
    import numpy as np
    import torch
    import triton
    from rdna3_fastmm.generated import rank7_2x2x2, rank49_4x4x4

    modules = {"rank7": (rank7_2x2x2, 2, 7), "rank49": (rank49_4x4x4, 4, 49)}
    record: dict = {"generator": "reference generated Triton kernels (FP16 mm path), TRITON_INTERPRET=1",
                    "triton": triton.__version__, "torch": torch.__version__, "cases": []}
    arrays: dict = {}
    for name, shapes in CASES.items():
        module, s, rank = modules[name]
        for M, K, N in shapes:
            bm, bk, bn = -(-M // s), -(-K // s), -(-N // s)
            A = randn_fp16((M, K), 0)
            B = randn_fp16((K, N), 1)
            L = torch.empty((rank, bm, bk), dtype=torch.float16)
            module.left_transform_kernel[(triton.cdiv(bm * bk, BLOCK_ELEMENTS),)](
                A, L, M, K, bm, bk, bm, bk, BLOCK_ELEMENTS)
            R = torch.empty((rank, bk, bn), dtype=torch.float16)
            module.right_transform_kernel[(triton.cdiv(bk * bn, BLOCK_ELEMENTS),)](
                B, R, K, N, bk, bn, bk, bn, BLOCK_ELEMENTS)
            W = B.t().contiguous()
            Rw = torch.empty((rank, bk, bn), dtype=torch.float16)
            module.right_transform_weight_kernel[(triton.cdiv(bk, 4), triton.cdiv(bn, 64))](
                W, Rw, N, K, bk, bn, 4, 64)
            P = random_products(rank, bm, bn, seed=3)
            bias = randn_fp16((N,), 2, 0.02)
            grid = (triton.cdiv(bm * bn, BLOCK_ELEMENTS),)
            C = torch.zeros((M, N), dtype=torch.float16)
            module.output_transform_kernel[grid](P, C, bm, bn, M, N, bm, bn, BLOCK_ELEMENTS)
            Cb = torch.zeros((M, N), dtype=torch.float16)
            module.output_transform_bias_kernel[grid](P, Cb, bias, bm, bn, M, N, bm, bn, BLOCK_ELEMENTS)
            record["cases"].append({
                "scheme": name, "shape": [M, K, N], "seeds": {"A": 0, "B": 1, "P": 3, "bias": 2},
                "inputs": {"A": digest(A), "B": digest(B), "P": digest(P), "bias": digest(bias)},
                "left": digest(L), "right": digest(R), "weight": digest(Rw), "output": digest(C),
                "output_bias": digest(Cb)})
            if (M, K, N) in SMALL:
                key = f"{name}_{M}x{K}x{N}"
                arrays[key + "_left"] = L.view(torch.int16).numpy()
                arrays[key + "_right"] = R.view(torch.int16).numpy()
                arrays[key + "_output"] = C.view(torch.int16).numpy()
                arrays[key + "_output_bias"] = Cb.view(torch.int16).numpy()
            print(name, (M, K, N), "done", flush=True)
    (HERE / "golden_mm.json").write_text(json.dumps(record, indent=1) + "\n")
    np.savez_compressed(HERE / "golden_mm.npz", **arrays)


if __name__ == "__main__":
    main()
