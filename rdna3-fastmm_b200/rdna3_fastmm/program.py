"""Straight-line linear programs: the common form of every transform.

Each side of a scheme (left, right, output) is turned into a
:class:`LinearProgram`: an ordered list of steps over numbered signals.
Signals ``0..inputs-1`` are the input blocks; every ``gate`` step defines the
next signal; every ``output`` step names a program output and the expression
that produces it.  Expressions are trees that keep the exact association of
the certificate, because the CUDA transforms must reproduce the reference's
floating-point operation order bit for bit:

* ``("sig", i)``                 signal ``i``
* ``("neg", e)``                 ``0 - e`` (one rounding; a zero operand gives
  +0, the signed-zero behaviour of the reference's Triton unary minus)
* ``("add", a, b)``/``("sub", a, b)``  ``a + b`` / ``a - b`` (one rounding)
* ``("scale", e, c)``            ``e * c`` for a dyadic rational ``c``
  (exact in binary floating point away from under/overflow, so ``e / 2`` and
  ``e * 0.5`` round identically)

The reduced-circuit association rule (first term, optionally negated, then
left-to-right ``+``/``-``) follows ``tools/generate_triton_scheme.py:70-79``
of the reference; the step order follows its schedulers
(``tools/generate_triton_scheme.py:27-67`` for reduced circuits,
``tools/generate_slp_triton_scheme.py:15-47`` for SLPs).
"""

from __future__ import annotations

from dataclasses import dataclass
from fractions import Fraction
from typing import Sequence, Union

Expr = tuple  # see module docstring

__all__ = ["Expr", "Step", "LinearProgram", "expr_signals", "expr_coefficients"]


@dataclass(frozen=True)
class Step:
    kind: str  # "gate" | "output"
    index: int  # gate number, or output number
    expr: Expr


@dataclass(frozen=True)
class LinearProgram:
    """``inputs`` signals in, ``outputs`` values out, evaluated by ``steps``."""

    inputs: int
    outputs: int
    steps: tuple[Step, ...]

    @property
    def gates(self) -> int:
        return sum(1 for s in self.steps if s.kind == "gate")

    def signal_count(self) -> int:
        return self.inputs + self.gates

    def coefficients(self) -> list[list[Fraction]]:
        """Dense coefficient rows (over the inputs) of every output, in order."""
        rows: list[list[Fraction]] = [
            [Fraction(int(j == i)) for j in range(self.inputs)] for i in range(self.inputs)
        ]
        out: list[list[Fraction] | None] = [None] * self.outputs
        for step in self.steps:
            value = expr_coefficients(step.expr, rows, self.inputs)
            if step.kind == "gate":
                if step.index != len(rows) - self.inputs:
                    raise ValueError("gate steps must be numbered in order")
                rows.append(value)
            else:
                if out[step.index] is not None:
                    raise ValueError(f"output {step.index} defined twice")
                out[step.index] = value
        if any(row is None for row in out):
            raise ValueError("program does not define every output")
        return [row for row in out if row is not None]

    def operation_counts(self) -> tuple[int, int]:
        """(additions, non-unit scalings) over every step."""
        adds = scales = 0
        stack = [s.expr for s in self.steps]
        while stack:
            e = stack.pop()
            op = e[0]
            if op in ("add", "sub"):
                adds += 1
                stack.extend((e[1], e[2]))
            elif op == "neg":
                stack.append(e[1])
            elif op == "scale":
                scales += int(abs(e[2]) != 1)
                stack.append(e[1])
        return adds, scales


def expr_signals(expr: Expr) -> list[int]:
    """Signals an expression reads, in first-use (left-to-right) order."""
    seen: list[int] = []

    def walk(e: Expr) -> None:
        if e[0] == "sig":
            if e[1] not in seen:
                seen.append(e[1])
        elif e[0] in ("add", "sub"):
            walk(e[1])
            walk(e[2])
        else:
            walk(e[1])

    walk(expr)
    return seen


def expr_coefficients(
    expr: Expr, rows: Sequence[Sequence[Fraction]], width: int
) -> list[Fraction]:
    op = expr[0]
    if op == "sig":
        return list(rows[expr[1]])
    if op == "neg":
        return [-c for c in expr_coefficients(expr[1], rows, width)]
    if op == "scale":
        k = Fraction(expr[2])
        return [k * c for c in expr_coefficients(expr[1], rows, width)]
    a = expr_coefficients(expr[1], rows, width)
    b = expr_coefficients(expr[2], rows, width)
    sign = 1 if op == "add" else -1
    return [x + sign * y for x, y in zip(a, b)]


def terms_to_expr(terms: Sequence[dict]) -> Expr:
    """Signed-unit term list -> left-associated expression tree."""
    first = terms[0]
    expr: Union[Expr, None] = ("sig", first["index"])
    if first["value"] == -1:
        expr = ("neg", expr)
    for term in terms[1:]:
        expr = ("add" if term["value"] == 1 else "sub", expr, ("sig", term["index"]))
    return expr
