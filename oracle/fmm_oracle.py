"""CPU oracle for the reduced-rank BF16 linear path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The shipped path (``rdna3_fastmm``) never imports, links or calls
anything under ``oracle/``.

It restates, in numpy, the algorithm of chelokot/rdna3-fastmm for one
``F.linear(x, weight, bias)`` call with a ``<s,s,s>`` rank-R scheme:

1. block split with zero padding, ``bm = ceil(M/s)`` etc.
   (``src/rdna3_fastmm/runtime.py:56-89``);
2. left transform ``L_r = sum_q U[r,q] A_q`` in FP32, stored FP16
   (``src/rdna3_fastmm/generated/*.py`` ``left_transform_kernel``;
   generator ``tools/generate_triton_scheme.py:82-233``);
3. weight transform ``R_r = sum_q V[r,q] B_q`` with ``B = weight^T`` read from
   the native ``weight[N, K]`` (``right_transform_weight_kernel``; generator
   ``tools/generate_triton_scheme.py:240-337``), stored FP16 as ``[R, bk, bn]``;
4. leaf products ``P_r = L_r @ R_r`` accumulated wide and stored FP16
   (``torch.bmm`` at ``src/rdna3_fastmm/runtime.py:728-732``);
5. output transform ``C_o = sum_r W[o,r] P_r (+ bias)`` in FP32 with a BF16
   round-to-nearest-even store (``output_transform{,_bias}_kernel``); for the
   FP16 square rank-343 scheme, a +-1 coefficient sum with an FP16 store
   (``generated/rank343_8x8x8.py`` ``output_transform_mfma_kernel``).

Planes are FP16 by default.  ``planes="bf16"`` gives the reference's
``(bfloat16, bfloat16)`` precision pair of ``Rank49Plan``
(``src/rdna3_fastmm/runtime.py:852-858``): the same FP32 arithmetic, with
every plane and product rounded to BF16 (nearest even) instead; BF16 planes
are returned as float32 arrays holding BF16 values.

Every gate and output is evaluated with the association written in the
certificate (left to right over signed terms for reduced circuits, the parsed
expression tree for SLP lines), which is the order the reference kernels use,
so FP16 planes agree bit for bit.  The evaluation here is written
independently of the product's scheme layer: it interprets the certificate
files directly.
"""

from __future__ import annotations

import ast
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

CERTIFICATES = (
    Path(__file__).resolve().parent.parent / "rdna3-fastmm_b200" / "rdna3_fastmm" / "certificates"
)

SCHEMES = {
    "rank7": ("reduced", "2x2x2_rank7_15add", 2, 7),
    "rank49": ("reduced", "4x4x4_rank49_159add", 4, 49),
    "rank48": ("slp", "4x4x4_rank48_accurate", 4, 48),
    "rank343": ("reduced", "8x8x8_rank343_1661add", 8, 343),
}
# schemes whose output side is a +-1 coefficient sum rather than the circuit
# (the reference reconstructs rank 343 with a matrix product against the
# expanded coefficients: generated/rank343_8x8x8.py output_transform_mfma_kernel)
COEFFICIENT_SUM_OUTPUT = frozenset({"rank343"})


# ---------------------------------------------------------------- number formats
def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.float32(np.nan)
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bfloat16-representable float32 values -> uint16 bit patterns."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- certificates
class _Circuit:
    """One side of a scheme: evaluate(inputs) -> outputs, certificate order."""

    def __init__(self, kind: str, payload, inputs: int, outputs: int):
        self.kind = kind
        self.payload = payload
        self.inputs = inputs
        self.outputs = outputs

    def evaluate(self, signals: list[np.ndarray]) -> list[np.ndarray]:
        sig = list(signals)
        if self.kind == "reduced":
            gates, exprs = self.payload

            def combine(terms):
                first = sig[terms[0]["index"]]
                # a leading minus is ``0 - x`` (Triton's unary minus), which
                # gives +0 for a zero operand
                acc = first if terms[0]["value"] == 1 else np.float32(0.0) - first
                for t in terms[1:]:
                    acc = acc + sig[t["index"]] if t["value"] == 1 else acc - sig[t["index"]]
                return acc

            for g in gates:
                sig.append(combine(g))
            return [combine(e) for e in exprs]
        # dyadic SLP: evaluate every line's expression tree on float32 arrays
        lines, order = self.payload
        env = {f"i{k}": v for k, v in enumerate(signals)}
        outs: dict[int, np.ndarray] = {}
        for target, tree in lines:
            env[target] = _eval_slp(tree, env)
            if target.startswith("o") and target[1:].isdigit():
                outs[int(target[1:])] = env[target]
        return [outs[order[k]] for k in range(self.outputs)]


def _eval_slp(node, env):
    if isinstance(node, ast.Name):
        return env[node.id]
    if isinstance(node, ast.Constant):
        return np.float32(node.value)
    a, b = _eval_slp(node.left, env), _eval_slp(node.right, env)
    if isinstance(node.op, ast.Add):
        return a + b
    if isinstance(node.op, ast.Sub):
        return a - b
    if isinstance(node.op, ast.Mult):
        return np.float32(a * b) if np.isscalar(a) and np.isscalar(b) else a * b
    if isinstance(node.op, ast.Div):
        return a / b
    raise ValueError("unsupported SLP operator")


@lru_cache(maxsize=None)
def scheme_circuits(name: str):
    """(size, rank, left, right, output) with row-major block numbering:
    left input q = A block (q//s, q%s); right input q = B block (q//s, q%s);
    output o = C block (o//s, o%s)."""
    kind, folder, s, rank = SCHEMES[name]
    base = CERTIFICATES / folder
    if kind == "reduced":
        cert = json.loads((base / "certificate.json").read_text())
        left = _Circuit("reduced", (cert["u_fresh"], cert["u"]), s * s, rank)
        right = _Circuit("reduced", (cert["v_fresh"], cert["v"]), s * s, rank)
        # certificate outputs are column-major C blocks; reorder to row-major
        w = cert["w"]
        row_major = [w[(o % s) * s + (o // s)] for o in range(s * s)]
        output = _Circuit("reduced", (cert["w_fresh"], row_major), rank, s * s)
        return s, rank, left, right, output

    def program(file: str, n_in: int, n_out: int) -> _Circuit:
        lines = []
        for raw in (base / file).read_text().splitlines():
            raw = raw.strip()
            if raw:
                target, body = raw[:-1].split(":=", 1)
                lines.append((target, ast.parse(body, mode="eval").body))
        return _Circuit("slp", (lines, list(range(n_out))), n_in, n_out)

    return (s, rank, program("left.slp", s * s, rank), program("right.slp", s * s, rank),
            program("output.slp", rank, s * s))


# ---------------------------------------------------------------- the path
def block_dims(M: int, K: int, N: int, s: int) -> tuple[int, int, int]:
    return -(-M // s), -(-K // s), -(-N // s)


def _blocks(src: np.ndarray, s: int, bh: int, bw: int) -> list[np.ndarray]:
    """Row-major list of the s*s zero-padded (bh, bw) blocks of ``src``."""
    padded = np.zeros((s * bh, s * bw), dtype=np.float32)
    padded[: src.shape[0], : src.shape[1]] = src
    return [padded[i * bh:(i + 1) * bh, j * bw:(j + 1) * bw] for i in range(s) for j in range(s)]


def round_plane(x: np.ndarray, planes: str = "fp16") -> np.ndarray:
    """FP32 plane values rounded to the plane format (nearest even): float16,
    or float32 holding BF16 values for ``planes="bf16"``."""
    if planes == "fp16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    if planes == "bf16":
        return bf16_round(np.asarray(x, dtype=np.float32))
    raise ValueError(f"unknown plane format {planes!r}")


def left_transform(name: str, A: np.ndarray, planes: str = "fp16") -> np.ndarray:
    """A [M, K] (bf16 values as float32) -> L [R, bm, bk] planes."""
    s, rank, left, _, _ = scheme_circuits(name)
    M, K = A.shape
    bm, bk = -(-M // s), -(-K // s)
    outs = left.evaluate(_blocks(A.astype(np.float32), s, bm, bk))
    return np.stack([round_plane(o, planes) for o in outs])


def weight_transform(name: str, W: np.ndarray, planes: str = "fp16") -> np.ndarray:
    """weight [N, K] -> R [R, bk, bn] planes (transform of B = weight^T)."""
    s, rank, _, right, _ = scheme_circuits(name)
    B = np.ascontiguousarray(W.astype(np.float32).T)
    K, N = B.shape
    bk, bn = -(-K // s), -(-N // s)
    outs = right.evaluate(_blocks(B, s, bk, bn))
    return np.stack([round_plane(o, planes) for o in outs])


def leaf_products(L: np.ndarray, R: np.ndarray, planes: str = "fp16") -> np.ndarray:
    """Planes -> products in the plane format, accumulated in float64 then
    rounded (through float32 for BF16)."""
    return round_plane(np.matmul(L.astype(np.float64), R.astype(np.float64)), planes)


@lru_cache(maxsize=None)
def output_coefficients(name: str) -> np.ndarray:
    """Expanded output map W[o, r] (row-major C blocks), exact integers: the
    output circuit evaluated on unit vectors."""
    s, rank, _, _, output = scheme_circuits(name)
    units = [np.eye(rank, dtype=np.float64)[r] for r in range(rank)]
    return np.stack(output.evaluate(units)).astype(np.int64)


def _coefficient_sum(name: str, P: np.ndarray) -> list[np.ndarray]:
    """``C_o = sum_r W[o, r] P_r`` accumulated in float32 from +0 in ascending
    r, one add or subtract per +-1 coefficient (the order the B200 kernel
    uses; the reference's matrix-product reconstruction leaves the order to
    the hardware)."""
    W = output_coefficients(name)
    acc = [np.zeros(P.shape[1:], dtype=np.float32) for _ in range(W.shape[0])]
    for r in range(W.shape[1]):
        p = P[r].astype(np.float32)
        for o in np.nonzero(W[:, r])[0]:
            acc[o] = acc[o] + p if W[o, r] > 0 else acc[o] - p
    return acc


def output_transform(name: str, P: np.ndarray, M: int, N: int,
                     bias: np.ndarray | None = None, out_dtype: str = "bf16") -> np.ndarray:
    """P [R, bm, bn] (float16, or float32 holding BF16 products) -> C [M, N]
    as float32 holding bf16 values
    (``out_dtype="fp16"``: FP16 values, the reference's FP16-plan output)."""
    s, rank, _, _, output = scheme_circuits(name)
    bm, bn = P.shape[1], P.shape[2]
    if name in COEFFICIENT_SUM_OUTPUT:
        outs = _coefficient_sum(name, P)
    else:
        outs = output.evaluate([P[r].astype(np.float32) for r in range(rank)])
    C = np.zeros((s * bm, s * bn), dtype=np.float32)
    for o, value in enumerate(outs):
        br, bc = divmod(o, s)
        if bias is not None:
            b = np.zeros(s * bn, dtype=np.float32)
            b[: bias.shape[0]] = bias.astype(np.float32)
            value = value + b[bc * bn:(bc + 1) * bn][None, :]
        C[br * bm:(br + 1) * bm, bc * bn:(bc + 1) * bn] = value
    if out_dtype == "fp16":
        return C[:M, :N].astype(np.float16).astype(np.float32)
    return bf16_round(C[:M, :N])


def linear(name: str, A: np.ndarray, W: np.ndarray, bias: np.ndarray | None = None,
           products=leaf_products, planes: str = "fp16") -> np.ndarray:
    """Whole path: ``F.linear(A, W, bias)`` as the reduced-rank algorithm."""
    L = left_transform(name, A, planes)
    R = weight_transform(name, W, planes)
    P = products(L, R) if planes == "fp16" else products(L, R, planes)
    return output_transform(name, P, A.shape[0], W.shape[0], bias)


def right_transform(name: str, B: np.ndarray) -> np.ndarray:
    """B [K, N] (the plain-mm right operand) -> R [R, bk, bn] float16."""
    return weight_transform(name, np.ascontiguousarray(np.asarray(B, dtype=np.float32).T))


def matmul(name: str, A: np.ndarray, B: np.ndarray, products=leaf_products) -> np.ndarray:
    """Plain ``A @ B`` with FP16 inputs and output (the mm API)."""
    L = left_transform(name, A)
    R = right_transform(name, B)
    return output_transform(name, products(L, R), A.shape[0], B.shape[1], None, "fp16")


def relative_l2(candidate: np.ndarray, reference: np.ndarray) -> float:
    c = np.asarray(candidate, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    return float(np.linalg.norm(c - r) / np.linalg.norm(r))
