"""CUDA generator: verified linear programs -> sm_100a device code.

For every scheme side (left, right, output) this emits a struct with a
``run`` member template that evaluates the program on a vector type ``V``
through caller-supplied ``in(q)`` and ``out(o, value)`` functors.  The block
addressing, vector width, bounds handling and stores live in the hand-written
kernels (``csrc/transforms.cuh``); the generated part only fixes *which*
signals are combined and *in what order*, one ``vadd``/``vsub``/``vneg``/
``vscale`` per certificate operation, so that each FP32 rounding happens
exactly where the reference's generated kernels round
(``src/rdna3_fastmm/generated/rank{7_2x2x2,48_4x4x4,49_4x4x4,343_8x8x8}.py``).

The output file is checked in; ``tests/test_codegen.py`` regenerates it and
requires byte equality, like the reference's own generator-determinism tests
(``tests/test_slp.py:58-59``).

Run ``python -m rdna3_fastmm.codegen`` to rewrite ``csrc/generated``.
"""

from __future__ import annotations

from fractions import Fraction
from pathlib import Path

from .program import Expr, LinearProgram, expr_signals
from .schemes import SCHEME_NAMES, SQUARE_SCHEME_NAMES, get_scheme

GENERATED_HEADER = (
    Path(__file__).resolve().parent.parent / "csrc" / "generated" / "fmm_schemes.cuh"
)


def _literal(value: Fraction) -> str:
    as_float = float(value)
    if Fraction(as_float) != value:
        raise ValueError(f"scale {value} is not exactly representable")
    text = repr(as_float)
    return text + "f"


def _render(expr: Expr) -> str:
    op = expr[0]
    if op == "sig":
        return f"s{expr[1]}"
    if op == "neg":
        return f"vneg({_render(expr[1])})"
    if op == "add":
        return f"vadd({_render(expr[1])}, {_render(expr[2])})"
    if op == "sub":
        return f"vsub({_render(expr[1])}, {_render(expr[2])})"
    if op == "scale":
        return f"vscale({_render(expr[1])}, {_literal(Fraction(expr[2]))})"
    raise ValueError(f"unknown expression {op}")


def _program_body(program: LinearProgram) -> list[str]:
    lines: list[str] = []
    loaded: set[int] = set()
    for step in program.steps:
        for sig in expr_signals(step.expr):
            if sig < program.inputs and sig not in loaded:
                lines.append(f"    const V s{sig} = in({sig});")
                loaded.add(sig)
        value = _render(step.expr)
        if step.kind == "gate":
            lines.append(f"    const V s{program.inputs + step.index} = {value};")
        else:
            lines.append(f"    out({step.index}, {value});")
    return lines


def _struct(name: str, program: LinearProgram) -> str:
    body = "\n".join(_program_body(program))
    return (
        f"struct {name} {{\n"
        f"  static constexpr int kInputs = {program.inputs};\n"
        f"  static constexpr int kOutputs = {program.outputs};\n"
        f"  template <class V, class In, class Out>\n"
        f"  static __device__ __forceinline__ void run(const In& in, const Out& out) {{\n"
        f"{body}\n"
        f"  }}\n"
        f"}};\n"
    )


def _output_sum_struct(name: str, program: LinearProgram, group: int = 8) -> str:
    """Output side as a coefficient sum: ``acc[o] += W[o][r] * p_r`` for r in
    ascending order, one FP32 add or subtract per nonzero (all coefficients
    are +-1).  Used where the product count makes a register-resident circuit
    impractical (rank 343: 343 inputs, 527 gates); the reference reconstructs
    this scheme with a tensor-core product against the same coefficient
    matrix, whose summation order is unspecified, so parity for this side is
    by tolerance.  Products are read ``group`` at a time so their loads are
    in flight together."""
    rows = program.coefficients()
    columns: list[list[tuple[int, int]]] = [[] for _ in range(program.inputs)]
    for o, row in enumerate(rows):
        for r, c in enumerate(row):
            if c == 0:
                continue
            if c not in (1, -1):
                raise ValueError("the coefficient-sum output needs +-1 coefficients")
            columns[r].append((o, int(c)))
    body: list[str] = []
    for start in range(0, program.inputs, group):
        stop = min(start + group, program.inputs)
        body.append("    {")
        for r in range(start, stop):
            body.append(f"      const V p{r} = in({r});")
        for r in range(start, stop):
            for o, c in columns[r]:
                op = "vadd" if c > 0 else "vsub"
                body.append(f"      acc[{o}] = {op}(acc[{o}], p{r});")
        body.append("    }")
    return (
        f"struct {name} {{\n"
        f"  static constexpr int kInputs = {program.inputs};\n"
        f"  static constexpr int kOutputs = {program.outputs};\n"
        f"  template <class V, class In>\n"
        f"  static __device__ __forceinline__ void accumulate(const In& in, V (&acc)[{program.outputs}]) {{\n"
        + "\n".join(body) + "\n"
        f"  }}\n"
        f"}};\n"
    )


def generate() -> str:
    parts = [
        "// Generated by rdna3_fastmm/codegen.py from the vendored certificates.",
        "// Do not edit: regenerate with `python -m rdna3_fastmm.codegen`.",
        "//",
        "// Each struct evaluates one side of a verified block scheme on a vector",
        "// type V; vadd/vsub/vneg/vscale are single FP32 roundings supplied by",
        "// csrc/transforms.cuh.",
        "#pragma once",
        "",
        "namespace fmm {",
        "namespace gen {",
        "",
    ]
    for name in SCHEME_NAMES + SQUARE_SCHEME_NAMES:
        scheme = get_scheme(name)
        camel = name.capitalize()
        parts.append(f"// {scheme.algorithm}: <{scheme.size},{scheme.size},{scheme.size}> rank {scheme.rank}")
        parts.append(f"// certificate sha256 {scheme.certificate_sha256}")
        parts.append(f"constexpr int k{camel}Size = {scheme.size};")
        parts.append(f"constexpr int k{camel}Rank = {scheme.rank};")
        parts.append("")
        parts.append(_struct(f"{camel}Left", scheme.left))
        parts.append(_struct(f"{camel}Right", scheme.right))
        if name in SQUARE_SCHEME_NAMES:
            parts.append(_output_sum_struct(f"{camel}OutputSum", scheme.output))
        else:
            parts.append(_struct(f"{camel}Output", scheme.output))
    parts.append("}  // namespace gen")
    parts.append("}  // namespace fmm")
    return "\n".join(parts) + "\n"


def main() -> None:
    GENERATED_HEADER.parent.mkdir(parents=True, exist_ok=True)
    GENERATED_HEADER.write_text(generate())


if __name__ == "__main__":
    main()
