"""Generate the golden fixtures by running the REFERENCE's own kernels.

Run once in a container that has chelokot/rdna3-fastmm checked out (the path
is given by ``--reference``; it is never read at test time):

    python tests/golden/make_golden.py --reference <path-to-reference>

The reference's generated Triton kernels
(``src/rdna3_fastmm/generated/rank{7_2x2x2,48_4x4x4,49_4x4x4}.py``) are run on
CPU tensors under ``TRITON_INTERPRET=1``.  The interpreter truncates FP32 ->
BF16 on store, so the output-transform kernels store into an FP32 buffer and
the BF16 round-to-nearest-even is done by ``Tensor.to(torch.bfloat16)``
(FP16 stores are correctly rounded and are used as-is).

Writes ``golden.json`` (SHA-256 digests of every plane for every case) and
``golden_small.npz`` (full arrays for the small cases).
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

from inputs import digest, make_linear_inputs, random_products  # noqa: E402

CASES = {
    "rank7": [(5, 6, 7), (17, 19, 23), (257, 263, 269), (512, 1024, 1024)],
    "rank49": [(5, 6, 7), (17, 19, 23), (257, 263, 269)],
    "rank48": [(5, 6, 7), (17, 19, 23), (257, 263, 269)],
}
SMALL = {(5, 6, 7), (17, 19, 23)}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference / "src"))
    import torch
    import triton
    from rdna3_fastmm.generated import rank7_2x2x2, rank48_4x4x4, rank49_4x4x4

    modules = {"rank7": (rank7_2x2x2, 2, 7), "rank49": (rank49_4x4x4, 4, 49),
               "rank48": (rank48_4x4x4, 4, 48)}
    record: dict = {"generator": "reference generated Triton kernels, TRITON_INTERPRET=1",
                    "triton": triton.__version__, "torch": torch.__version__, "cases": []}
    arrays: dict = {}
    for name, shapes in CASES.items():
        module, s, rank = modules[name]
        for M, K, N in shapes:
            bm, bk, bn = -(-M // s), -(-K // s), -(-N // s)
            A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=True)
            L = torch.empty((rank, bm, bk), dtype=torch.float16)
            module.left_transform_kernel[(triton.cdiv(bm * bk, 256),)](
                A, L, M, K, bm, bk, bm, bk, 256)
            Rw = torch.empty((rank, bk, bn), dtype=torch.float16)
            module.right_transform_weight_kernel[(triton.cdiv(bk, 4), triton.cdiv(bn, 64))](
                W, Rw, N, K, bk, bn, 4, 64)
            P = random_products(rank, bm, bn, seed=3)
            outputs = {}
            for with_bias in (False, True):
                C32 = torch.zeros((M, N), dtype=torch.float32)
                grid = (triton.cdiv(bm * bn, 256),)
                if with_bias:
                    module.output_transform_bias_kernel[grid](P, C32, bias, bm, bn, M, N, bm, bn, 256)
                else:
                    module.output_transform_kernel[grid](P, C32, bm, bn, M, N, bm, bn, 256)
                outputs[with_bias] = C32.to(torch.bfloat16)
            case = {"scheme": name, "shape": [M, K, N], "seed": 0, "product_seed": 3,
                    "inputs": {"A": digest(A), "W": digest(W), "bias": digest(bias),
                               "P": digest(P)},
                    "left": digest(L), "weight": digest(Rw),
                    "output": digest(outputs[False]), "output_bias": digest(outputs[True])}
            record["cases"].append(case)
            if (M, K, N) in SMALL:
                key = f"{name}_{M}x{K}x{N}"
                arrays[key + "_left"] = L.view(torch.int16).numpy()
                arrays[key + "_weight"] = Rw.view(torch.int16).numpy()
                arrays[key + "_output"] = outputs[False].view(torch.int16).numpy()
                arrays[key + "_output_bias"] = outputs[True].view(torch.int16).numpy()
            print(name, (M, K, N), "done", flush=True)
        # exact small integer product (the reference's GPU known-answer test shape)
        g = torch.Generator().manual_seed(11)
        A = torch.randint(-2, 3, (5, 6), generator=g).to(torch.bfloat16)
        W = torch.randint(-2, 3, (7, 6), generator=g).to(torch.bfloat16)
        bm, bk, bn = -(-5 // s), -(-6 // s), -(-7 // s)
        L = torch.empty((rank, bm, bk), dtype=torch.float16)
        module.left_transform_kernel[(triton.cdiv(bm * bk, 256),)](A, L, 5, 6, bm, bk, bm, bk, 256)
        Rw = torch.empty((rank, bk, bn), dtype=torch.float16)
        module.right_transform_weight_kernel[(triton.cdiv(bk, 4), triton.cdiv(bn, 64))](
            W, Rw, 7, 6, bk, bn, 4, 64)
        P = torch.bmm(L.float(), Rw.float()).half()
        C32 = torch.zeros((5, 7), dtype=torch.float32)
        module.output_transform_kernel[(triton.cdiv(bm * bn, 256),)](P, C32, bm, bn, 5, 7, bm, bn, 256)
        key = f"{name}_exact"
        arrays[key + "_A"] = A.view(torch.int16).numpy()
        arrays[key + "_W"] = W.view(torch.int16).numpy()
        arrays[key + "_C"] = C32.to(torch.bfloat16).view(torch.int16).numpy()
    (HERE / "golden.json").write_text(json.dumps(record, indent=1) + "\n")
    import numpy as np
    np.savez_compressed(HERE / "golden_small.npz", **arrays)


if __name__ == "__main__":
    main()
