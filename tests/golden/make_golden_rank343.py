"""Golden fixtures for the rank-343 <8,8,8> FP16 square scheme, made by running
the REFERENCE's own generated kernels.

Run once in a container that has chelokot/rdna3-fastmm checked out (never read
at test time):

    python tests/golden/make_golden_rank343.py --reference <path-to-reference>

``src/rdna3_fastmm/generated/rank343_8x8x8.py`` is run on CPU tensors under
``TRITON_INTERPRET=1``: ``left_transform_kernel`` on ``A[M, K]``,
``right_transform_kernel`` on ``B[K, N]`` (both FP16, the scheme's only
precision) and ``output_transform_mfma_kernel`` (FP16 products times the
+-1 coefficient matrix, FP32 accumulation) on seeded random products, stored
into an FP32 buffer and rounded to FP16 by torch.  Launch parameters follow
the reference plan (``runtime.py:906-962``).  Writes ``golden_rank343.json``
(digests) and ``golden_rank343.npz`` (full arrays).
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

from inputs import digest, random_products, randn_fp16  # noqa: E402

SHAPES = [(5, 6, 7), (17, 19, 23), (67, 71, 73)]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference / "src"))
    import numpy as np
    import torch
    import triton
    from rdna3_fastmm.generated import rank343_8x8x8 as module

    s, rank = 8, 343
    coefficients = torch.tensor(module.MFMA_OUTPUT_COEFFICIENTS, dtype=torch.float16)
    record: dict = {"generator": "reference rank343_8x8x8.py kernels, TRITON_INTERPRET=1",
                    "triton": triton.__version__, "torch": torch.__version__, "cases": []}
    arrays: dict = {}

    def run(A, B, P):
        M, K = A.shape
        N = B.shape[1]
        bm, bk, bn = -(-M // s), -(-K // s), -(-N // s)
        L = torch.empty((rank, bm, bk), dtype=torch.float16)
        module.left_transform_kernel[(triton.cdiv(bm * bk, 1024),)](A, L, M, K, bm, bk, bm, bk, 1024)
        R = torch.empty((rank, bk, bn), dtype=torch.float16)
        module.right_transform_kernel[(triton.cdiv(bk * bn, 512),)](B, R, K, N, bk, bn, bk, bn, 512)
        if P is None:
            P = torch.bmm(L.float(), R.float()).half()
        C32 = torch.zeros((M, N), dtype=torch.float32)
        module.output_transform_mfma_kernel[(triton.cdiv(bm * bn, 128),)](
            P, coefficients, C32, M, N, bm, bn, 128, 16)
        return L, R, P, C32.to(torch.float16)

    for M, K, N in SHAPES:
        A = randn_fp16((M, K), 0)
        B = randn_fp16((K, N), 1)
        bm, bn = -(-M // s), -(-N // s)
        P = random_products(rank, bm, bn, seed=3)
        L, R, _, C = run(A, B, P)
        key = f"rank343_{M}x{K}x{N}"
        record["cases"].append({"shape": [M, K, N], "A": digest(A), "B": digest(B), "P": digest(P),
                                "left": digest(L), "right": digest(R), "output": digest(C)})
        for name, t in (("left", L), ("right", R), ("output", C)):
            arrays[f"{key}_{name}"] = t.view(torch.int16).numpy()
        print((M, K, N), "done", flush=True)
    # exact small integer product (the reference's rank-343 known-answer shape)
    g = torch.Generator().manual_seed(17)
    A = torch.randint(-2, 3, (5, 6), generator=g).to(torch.float16)
    B = torch.randint(-2, 3, (6, 7), generator=g).to(torch.float16)
    _, _, _, C = run(A, B, None)
    arrays["rank343_exact_A"] = A.view(torch.int16).numpy()
    arrays["rank343_exact_B"] = B.view(torch.int16).numpy()
    arrays["rank343_exact_C"] = C.view(torch.int16).numpy()
    (HERE / "golden_rank343.json").write_text(json.dumps(record, indent=1) + "\n")
    np.savez_compressed(HERE / "golden_rank343.npz", **arrays)


if __name__ == "__main__":
    main()
