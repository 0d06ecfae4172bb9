"""Dyadic straight-line-program (SLP) certificates: parsing and exact checks.

An SLP certificate (used by the rank-48 ``<4,4,4>`` scheme) is a JSON
manifest naming three text programs ``u``, ``v`` and ``w``.  Each program line
is ``target:=expression;`` where the expression uses ``+``, ``-`` and
multiplication/division by integer constants over the inputs ``i0, i1, ...``
and every earlier target.  Targets ``o<k>`` are the program outputs.  Only
dyadic scalings (powers of two in the denominator) are accepted, so every
transform stays exact in binary floating point apart from rounding of sums.

Behaviour follows ``src/rdna3_fastmm/slp.py`` of chelokot/rdna3-fastmm:
expression rules (``:105-193``), program loading (``:196-263``), manifest
checks (``:286-360``), certificate digest (``:272-283``), and the Fraction
Brent-tensor check with a row-major output index (``:363-431``).  The SLP text
format and the digest recipe are those of the upstream certificate and of the
reference, and are kept identical so that certificate hashes agree.
"""

from __future__ import annotations

import ast
import hashlib
import json
import re
from dataclasses import dataclass
from fractions import Fraction
from pathlib import Path
from typing import Any

from .program import Expr, LinearProgram, Step

_NAME = re.compile(r"[A-Za-z][A-Za-z0-9_]*")

__all__ = [
    "SlpAssignment",
    "SlpProgram",
    "SlpCertificate",
    "SlpVerificationSummary",
    "load_slp_program",
    "load_slp_certificate",
    "verify_slp_certificate",
    "load_and_verify_slp_certificate",
]


@dataclass(frozen=True)
class SlpAssignment:
    target: str
    signal_index: int
    dependencies: tuple[int, ...]
    expr: Expr
    coefficients: tuple[Fraction, ...]
    additions: int
    scalings: int


@dataclass(frozen=True)
class SlpProgram:
    input_count: int
    output_count: int
    assignments: tuple[SlpAssignment, ...]
    output_signals: tuple[int, ...]
    output_coefficients: tuple[tuple[Fraction, ...], ...]
    additions: int
    scalings: int

    @property
    def operations(self) -> int:
        return self.additions + self.scalings

    def to_linear_program(self, output_index: dict[int, int] | None = None) -> LinearProgram:
        """Every assignment becomes a gate; each ``o<k>`` also emits output
        ``output_index[k]`` right after its gate (identity by default)."""
        steps: list[Step] = []
        for gate, a in enumerate(self.assignments):
            steps.append(Step("gate", gate, a.expr))
            if _output_number(a.target) is not None:
                k = _output_number(a.target)
                steps.append(
                    Step("output", k if output_index is None else output_index[k], ("sig", a.signal_index))
                )
        return LinearProgram(self.input_count, self.output_count, tuple(steps))


@dataclass(frozen=True)
class SlpCertificate:
    dimensions: tuple[int, int, int]
    rank: int
    left: SlpProgram
    right: SlpProgram
    output: SlpProgram
    sha256: str


@dataclass(frozen=True)
class SlpVerificationSummary:
    dimensions: tuple[int, int, int]
    rank: int
    additions: tuple[int, int, int]
    scalings: tuple[int, int, int]
    operations: tuple[int, int, int]
    tensor_entries: int
    sha256: str


def _output_number(target: str) -> int | None:
    if target.startswith("o") and target[1:].isdigit():
        return int(target[1:])
    return None


def _dyadic(value: Fraction) -> bool:
    d = value.denominator
    return d > 0 and (d & (d - 1)) == 0


class _Value:
    """Intermediate parse result: a scalar constant or a linear expression."""

    __slots__ = ("scalar", "coeffs", "expr", "deps", "adds", "scales")

    def __init__(self, scalar=None, coeffs=None, expr=None, deps=(), adds=0, scales=0):
        self.scalar = scalar
        self.coeffs = coeffs
        self.expr = expr
        self.deps = deps
        self.adds = adds
        self.scales = scales


def _merge(a: tuple[int, ...], b: tuple[int, ...]) -> tuple[int, ...]:
    out = list(a)
    for x in b:
        if x not in out:
            out.append(x)
    return tuple(out)


def _parse(node: ast.expr, env: dict[str, tuple[int, tuple[Fraction, ...]]]) -> _Value:
    if isinstance(node, ast.Name):
        if node.id not in env:
            raise ValueError(f"SLP references unavailable signal {node.id}")
        index, coeffs = env[node.id]
        return _Value(coeffs=coeffs, expr=("sig", index), deps=(index,))
    if isinstance(node, ast.Constant):
        if isinstance(node.value, bool) or not isinstance(node.value, int):
            raise ValueError("SLP constants must be integers")
        return _Value(scalar=Fraction(node.value))
    if not isinstance(node, ast.BinOp):
        raise ValueError(f"unsupported SLP expression {type(node).__name__}")
    left = _parse(node.left, env)
    right = _parse(node.right, env)
    deps = _merge(left.deps, right.deps)
    adds = left.adds + right.adds
    scales = left.scales + right.scales
    op = node.op
    if isinstance(op, (ast.Add, ast.Sub)):
        if left.coeffs is None or right.coeffs is None:
            raise ValueError("SLP additions require two linear expressions")
        sign = 1 if isinstance(op, ast.Add) else -1
        coeffs = tuple(x + sign * y for x, y in zip(left.coeffs, right.coeffs, strict=True))
        kind = "add" if sign == 1 else "sub"
        return _Value(coeffs=coeffs, expr=(kind, left.expr, right.expr), deps=deps,
                      adds=adds + 1, scales=scales)
    if isinstance(op, ast.Mult):
        if left.scalar is not None and right.coeffs is not None:
            k, linear = left.scalar, right
        elif right.scalar is not None and left.coeffs is not None:
            k, linear = right.scalar, left
        else:
            raise ValueError("SLP multiplication requires one scalar")
    elif isinstance(op, ast.Div):
        if left.coeffs is None or right.scalar is None or right.scalar == 0:
            raise ValueError("SLP division requires a linear expression and scalar")
        k, linear = Fraction(1) / right.scalar, left
    else:
        raise ValueError(f"unsupported SLP operator {type(op).__name__}")
    if not _dyadic(k):
        raise ValueError("SLP scaling must be dyadic")
    return _Value(coeffs=tuple(k * c for c in linear.coeffs), expr=("scale", linear.expr, k),
                  deps=deps, adds=adds, scales=scales + int(abs(k) != 1))


def load_slp_program(path: Path, input_count: int, output_count: int) -> SlpProgram:
    if input_count < 1 or output_count < 1:
        raise ValueError("SLP input and output counts must be positive")
    path = Path(path)
    env: dict[str, tuple[int, tuple[Fraction, ...]]] = {
        f"i{i}": (i, tuple(Fraction(int(j == i)) for j in range(input_count)))
        for i in range(input_count)
    }
    assignments: list[SlpAssignment] = []
    outputs: dict[int, SlpAssignment] = {}
    for number, raw in enumerate(path.read_text().splitlines(), 1):
        line = raw.strip()
        if not line:
            continue
        if not line.endswith(";") or line.count(":=") != 1:
            raise ValueError(f"{path}:{number}: invalid SLP assignment")
        target, body = line[:-1].split(":=", 1)
        if _NAME.fullmatch(target) is None:
            raise ValueError(f"{path}:{number}: invalid SLP target")
        if target in env:
            raise ValueError(f"{path}:{number}: duplicate SLP target {target}")
        try:
            tree = ast.parse(body, mode="eval").body
        except SyntaxError as error:
            raise ValueError(f"{path}:{number}: invalid SLP expression") from error
        value = _parse(tree, env)
        if value.coeffs is None:
            raise ValueError(f"{path}:{number}: SLP result must be linear")
        index = input_count + len(assignments)
        assignment = SlpAssignment(target, index, value.deps, value.expr, value.coeffs,
                                   value.adds, value.scales)
        assignments.append(assignment)
        env[target] = (index, value.coeffs)
        k = _output_number(target)
        if k is not None:
            if not 0 <= k < output_count:
                raise ValueError(f"{path}:{number}: output index {k} is out of range")
            outputs[k] = assignment
    if len(outputs) != output_count:
        missing = sorted(set(range(output_count)) - set(outputs))
        raise ValueError(f"{path}: missing SLP outputs {missing}")
    ordered = [outputs[k] for k in range(output_count)]
    return SlpProgram(
        input_count=input_count,
        output_count=output_count,
        assignments=tuple(assignments),
        output_signals=tuple(a.signal_index for a in ordered),
        output_coefficients=tuple(a.coefficients for a in ordered),
        additions=sum(a.additions for a in assignments),
        scalings=sum(a.scalings for a in assignments),
    )


def _certificate_digest(manifest: Path, programs: list[tuple[str, Path]]) -> str:
    digest = hashlib.sha256(manifest.read_bytes())
    for name, path in programs:
        digest.update(b"\0" + name.encode() + b"\0")
        digest.update(path.read_bytes())
    return digest.hexdigest()


def load_slp_certificate(manifest_path: Path) -> SlpCertificate:
    manifest_path = Path(manifest_path)
    data: Any = json.loads(manifest_path.read_text())
    if not isinstance(data, dict):
        raise ValueError("SLP certificate must be an object")
    if data.get("schema_version") != 1:
        raise ValueError("unsupported SLP certificate schema")
    dims, rank = data.get("n"), data.get("m")
    ok_dims = isinstance(dims, list) and len(dims) == 3 and all(
        isinstance(d, int) and not isinstance(d, bool) and d >= 1 for d in dims
    )
    ok_rank = isinstance(rank, int) and not isinstance(rank, bool) and rank >= 1
    if not (ok_dims and ok_rank):
        raise ValueError("invalid SLP dimensions or rank")
    if data.get("domain") != "dyadic-rational":
        raise ValueError("SLP certificate must use the dyadic-rational domain")
    if data.get("input_order") != "row-major":
        raise ValueError("SLP certificate inputs must be row-major")
    if data.get("output_order") != "row-major":
        raise ValueError("SLP certificate outputs must be row-major")
    programs, complexity = data.get("programs"), data.get("complexity")
    if not isinstance(programs, dict) or not isinstance(complexity, dict):
        raise ValueError("SLP certificate programs and complexity must be objects")
    folder = manifest_path.parent.resolve()
    paths: list[tuple[str, Path]] = []
    for name in ("u", "v", "w"):
        rel = programs.get(name)
        if not isinstance(rel, str) or not rel:
            raise ValueError(f"certificate {name} must be a nonempty string")
        full = (folder / rel).resolve()
        if full.parent != folder:
            raise ValueError("SLP program paths must stay inside the certificate")
        paths.append((name, full))
    n0, n1, n2 = dims
    left = load_slp_program(paths[0][1], n0 * n1, rank)
    right = load_slp_program(paths[1][1], n1 * n2, rank)
    output = load_slp_program(paths[2][1], rank, n0 * n2)
    for name, program in (("u", left), ("v", right), ("w", output)):
        declared = complexity.get(name)
        if isinstance(declared, bool) or not isinstance(declared, int) or declared != program.operations:
            raise ValueError(f"SLP {name} complexity does not match the manifest")
    return SlpCertificate((n0, n1, n2), rank, left, right, output,
                          _certificate_digest(manifest_path, paths))


def verify_slp_certificate(certificate: SlpCertificate) -> SlpVerificationSummary:
    n0, n1, n2 = certificate.dimensions
    entries: dict[tuple[int, int, int], Fraction] = {}
    for r in range(certificate.rank):
        us = [(i, c) for i, c in enumerate(certificate.left.output_coefficients[r]) if c]
        vs = [(j, c) for j, c in enumerate(certificate.right.output_coefficients[r]) if c]
        ws = [(o, certificate.output.output_coefficients[o][r]) for o in range(n0 * n2)
              if certificate.output.output_coefficients[o][r]]
        for i, a in us:
            for j, b in vs:
                for o, c in ws:
                    entries[(i, j, o)] = entries.get((i, j, o), Fraction(0)) + a * b * c
    entries = {k: v for k, v in entries.items() if v}
    expected = {
        (row * n1 + inner, inner * n2 + col, row * n2 + col): Fraction(1)
        for row in range(n0) for inner in range(n1) for col in range(n2)
    }
    if entries != expected:
        wrong = sum(entries.get(k, Fraction(0)) != expected.get(k, Fraction(0))
                    for k in entries.keys() | expected.keys())
        raise ValueError(f"SLP Brent tensor has {wrong} mismatches")
    progs = (certificate.left, certificate.right, certificate.output)
    return SlpVerificationSummary(
        dimensions=certificate.dimensions,
        rank=certificate.rank,
        additions=tuple(p.additions for p in progs),
        scalings=tuple(p.scalings for p in progs),
        operations=tuple(p.operations for p in progs),
        tensor_entries=len(entries),
        sha256=certificate.sha256,
    )


def load_and_verify_slp_certificate(manifest_path: Path) -> tuple[SlpCertificate, SlpVerificationSummary]:
    certificate = load_slp_certificate(manifest_path)
    return certificate, verify_slp_certificate(certificate)
