"""Reduced-circuit certificates: loading and exact (integer) verification.

A reduced circuit describes a bilinear ``<n0, n1, n2>`` matrix-multiplication
scheme of rank ``m`` as three signed addition circuits:

* ``u_fresh``/``u``: the left map from the ``n0*n1`` row-major blocks of A to
  the ``m`` left factors,
* ``v_fresh``/``v``: the right map from the ``n1*n2`` row-major blocks of B to
  the ``m`` right factors,
* ``w_fresh``/``w``: the output map from the ``m`` products to the ``n0*n2``
  blocks of C, numbered column-major (block ``(row, col)`` is output
  ``col*n0 + row``).

Each expression is a list of ``{"index": i, "value": +-1}`` terms over the
signals available so far (the inputs, then every fresh gate in order).

Behaviour follows ``src/rdna3_fastmm/certificate.py`` of chelokot/rdna3-fastmm:
expansion (``:59-76``), cost model (``:79-94``), term validation
(``:97-127``), header checks (``:130-150``), Brent-tensor check
(``:163-255``) and the expanded loader (``:269-292``).  The certificate file
format is the upstream FastMatrixMultiplication JSON format and must be read
as-is.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping, Sequence

Term = Mapping[str, int]
Expression = Sequence[Term]

__all__ = [
    "ExpandedScheme",
    "VerificationSummary",
    "expand_linear_map",
    "circuit_cost",
    "verify_reduced_scheme",
    "load_reduced_scheme",
    "load_expanded_scheme",
]


@dataclass(frozen=True)
class VerificationSummary:
    dimensions: tuple[int, int, int]
    rank: int
    additions: int
    side_additions: tuple[int, int, int]
    naive_additions: int
    tensor_entries: int


@dataclass(frozen=True)
class ExpandedScheme:
    """Dense integer coefficient maps of a verified scheme.

    ``left_coefficients[r][q]`` multiplies row-major A block ``q`` in left
    factor ``r``; ``right_coefficients[r][q]`` multiplies row-major B block
    ``q``; ``output_coefficients[o][r]`` multiplies product ``r`` in the
    row-major C block ``o``.
    """

    dimensions: tuple[int, int, int]
    rank: int
    left_coefficients: tuple[tuple[int, ...], ...]
    right_coefficients: tuple[tuple[int, ...], ...]
    output_coefficients: tuple[tuple[int, ...], ...]


def _is_int(value: Any) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


def _check_terms(
    side: str, expressions: Sequence[Expression], inputs: int, gates: int
) -> None:
    """Every term is a signed unit over a signal that already exists."""
    if not isinstance(expressions, list):
        raise ValueError(f"{side} expressions must be a list")
    for position, expression in enumerate(expressions):
        if not isinstance(expression, list):
            raise ValueError(f"{side} expression {position} must be a list")
        if len(expression) == 0:
            raise ValueError(f"{side} expression {position} is empty")
        # gate g may use inputs and gates < g; outputs may use every gate
        visible = inputs + min(position, gates)
        for term in expression:
            if not isinstance(term, dict):
                raise ValueError(f"{side} expression {position} has invalid term")
            index, value = term.get("index"), term.get("value")
            if not _is_int(index):
                raise ValueError(f"{side} expression {position} has invalid index")
            if index < 0 or index >= visible:
                raise ValueError(
                    f"{side} expression {position} references unavailable signal {index}"
                )
            if not _is_int(value) or value not in (1, -1):
                raise ValueError(f"{side} expression {position} has non-signed value")


def expand_linear_map(
    input_count: int, gates: Sequence[Expression], outputs: Sequence[Expression]
) -> list[list[int]]:
    """Dense coefficient rows (over the inputs) of every output expression."""
    rows: list[list[int]] = [
        [1 if j == i else 0 for j in range(input_count)] for i in range(input_count)
    ]

    def combine(expression: Expression) -> list[int]:
        acc = [0] * input_count
        for term in expression:
            source = rows[term["index"]]
            sign = term["value"]
            for j in range(input_count):
                acc[j] += sign * source[j]
        return acc

    for gate in gates:
        rows.append(combine(gate))
    return [combine(expression) for expression in outputs]


def circuit_cost(gates: Sequence[Expression], outputs: Sequence[Expression]) -> int:
    """Additions of a circuit: a k-term expression costs k-1."""
    return sum(max(len(e) - 1, 0) for e in list(gates) + list(outputs))


def _header(source: Mapping[str, Any]) -> tuple[int, int, int, int]:
    dims = source.get("n")
    if not isinstance(dims, list) or len(dims) != 3 or not all(
        _is_int(d) and d >= 1 for d in dims
    ):
        raise ValueError("scheme dimensions must be three positive integers")
    rank = source.get("m")
    if not _is_int(rank) or rank < 1:
        raise ValueError("scheme rank must be a positive integer")
    if source.get("z2") is not False:
        raise ValueError("certificate must explicitly define an integer, non-Z2 circuit")
    return dims[0], dims[1], dims[2], rank


def _brent_entries(
    u: Sequence[Sequence[int]],
    v: Sequence[Sequence[int]],
    w_by_term: Sequence[Sequence[int]],
) -> dict[tuple[int, int, int], int]:
    """Sum over terms of u (x) v (x) w, keeping only nonzero entries."""
    total: dict[tuple[int, int, int], int] = {}
    for ur, vr, wr in zip(u, v, w_by_term, strict=True):
        nu = [(i, c) for i, c in enumerate(ur) if c]
        nv = [(i, c) for i, c in enumerate(vr) if c]
        nw = [(i, c) for i, c in enumerate(wr) if c]
        for i, a in nu:
            for j, b in nv:
                for k, c in nw:
                    key = (i, j, k)
                    total[key] = total.get(key, 0) + a * b * c
    return {key: value for key, value in total.items() if value}


def _matmul_tensor(n0: int, n1: int, n2: int) -> dict[tuple[int, int, int], int]:
    """<n0,n1,n2> tensor with a column-major output index."""
    return {
        (row * n1 + inner, inner * n2 + col, col * n0 + row): 1
        for row in range(n0)
        for inner in range(n1)
        for col in range(n2)
    }


def verify_reduced_scheme(source: Mapping[str, Any]) -> VerificationSummary:
    """Check a reduced circuit exactly over the integers.

    Raises ``ValueError`` on malformed circuits, a wrong Brent tensor, or a
    declared complexity that does not match the circuit.
    """
    n0, n1, n2, rank = _header(source)
    sides = (
        ("u", n0 * n1, source["u_fresh"], source["u"]),
        ("v", n1 * n2, source["v_fresh"], source["v"]),
        ("w", rank, source["w_fresh"], source["w"]),
    )
    expanded = []
    costs = []
    for name, inputs, gates, outputs in sides:
        _check_terms(name, list(gates) + list(outputs), inputs, len(gates))
        expanded.append(expand_linear_map(inputs, gates, outputs))
        costs.append(circuit_cost(gates, outputs))
    u, v, w_columns = expanded
    if len(u) != rank or len(v) != rank:
        raise ValueError("input factor row count does not match rank")
    if len(w_columns) != n0 * n2:
        raise ValueError("output circuit row count does not match output size")
    w_by_term = [[w_columns[o][r] for o in range(n0 * n2)] for r in range(rank)]
    actual = _brent_entries(u, v, w_by_term)
    expected = _matmul_tensor(n0, n1, n2)
    if actual != expected:
        wrong = sum(
            actual.get(key, 0) != expected.get(key, 0) for key in actual.keys() | expected.keys()
        )
        raise ValueError(f"Brent tensor has {wrong} mismatched entries")
    nonzeros = sum(1 for factor in (u, v, w_by_term) for row in factor for c in row if c)
    naive = nonzeros - 2 * rank - n0 * n2
    declared = source.get("complexity")
    if declared is not None:
        if not isinstance(declared, dict):
            raise ValueError("declared complexity must be an object")
        if declared.get("reduced") != sum(costs):
            raise ValueError("declared reduced complexity is incorrect")
        if declared.get("naive") != naive:
            raise ValueError("declared naive complexity is incorrect")
    return VerificationSummary(
        dimensions=(n0, n1, n2),
        rank=rank,
        additions=sum(costs),
        side_additions=(costs[0], costs[1], costs[2]),
        naive_additions=naive,
        tensor_entries=len(actual),
    )


def load_reduced_scheme(path: Path) -> dict[str, Any]:
    raw = json.loads(Path(path).read_text())
    if not isinstance(raw, dict):
        raise ValueError("certificate must be a JSON object")
    for key in ("n", "m", "u_fresh", "v_fresh", "w_fresh", "u", "v", "w"):
        if key not in raw:
            raise ValueError("input is not a reduced scheme")
    return raw


def load_expanded_scheme(path: Path) -> ExpandedScheme:
    """Load, verify and expand a reduced circuit into dense coefficient maps."""
    source = load_reduced_scheme(path)
    summary = verify_reduced_scheme(source)
    n0, n1, n2 = summary.dimensions
    left = expand_linear_map(n0 * n1, source["u_fresh"], source["u"])
    right = expand_linear_map(n1 * n2, source["v_fresh"], source["v"])
    w_columns = expand_linear_map(summary.rank, source["w_fresh"], source["w"])
    # re-index the column-major output circuit into row-major C blocks
    output = [w_columns[col * n0 + row] for row in range(n0) for col in range(n2)]
    return ExpandedScheme(
        dimensions=summary.dimensions,
        rank=summary.rank,
        left_coefficients=tuple(tuple(r) for r in left),
        right_coefficients=tuple(tuple(r) for r in right),
        output_coefficients=tuple(tuple(r) for r in output),
    )
