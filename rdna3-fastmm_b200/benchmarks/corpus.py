"""GEMM case corpus (schema 1) for the per-case report runner.

Reads the corpus format of the reference's ``benchmarks/corpus.py``
(chelokot/rdna3-fastmm, loader ``:170-200``, case fields ``:21-47``): a JSON
object ``{schema_version: 1, name, operator: "torch.nn.functional.linear",
cases: [...]}`` whose cases carry ``id, model, workload, projection,
shape [M, K, N], input_output_dtype, compute_dtype, weight_layout "out_in",
bias, priority 1-3, evidence {kind, note, references}``.  Every object must
carry exactly its keys; ids must be unique.  A reference corpus file loads
unchanged; the default corpus here lists the B200 headline shapes.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

DEFAULT_CORPUS_PATH = Path(__file__).resolve().parent / "corpora" / "b200-headline.json"
DTYPE_NAMES = frozenset({"float16", "bfloat16"})
EVIDENCE_KINDS = frozenset({"architecture-derived", "locally-profiled"})
CASE_KEYS = frozenset({"id", "model", "workload", "projection", "shape", "input_output_dtype",
                       "compute_dtype", "weight_layout", "bias", "priority", "evidence"})


@dataclass(frozen=True)
class Evidence:
    kind: str
    note: str
    references: tuple[str, ...]


@dataclass(frozen=True)
class GemmCase:
    id: str
    model: str
    workload: str
    projection: str
    shape: tuple[int, int, int]
    input_output_dtype: str
    compute_dtype: str
    weight_layout: str
    bias: bool
    priority: int
    evidence: Evidence

    @property
    def rows(self) -> int:
        return self.shape[0]

    @property
    def inner(self) -> int:
        return self.shape[1]

    @property
    def columns(self) -> int:
        return self.shape[2]


@dataclass(frozen=True)
class GemmCorpus:
    schema_version: int
    name: str
    operator: str
    cases: tuple[GemmCase, ...]

    def case(self, case_id: str) -> GemmCase:
        for case in self.cases:
            if case.id == case_id:
                return case
        raise KeyError(f"no case {case_id!r} in corpus {self.name!r}")


class _Reader:
    """Typed field access with the JSON path in every error message."""

    def __init__(self, value: object, where: str, keys: frozenset[str]) -> None:
        if not isinstance(value, dict) or not all(isinstance(k, str) for k in value):
            raise ValueError(f"{where} must be an object with string keys")
        if value.keys() != keys:
            missing = sorted(keys - value.keys())
            extra = sorted(value.keys() - keys)
            raise ValueError(f"{where} has invalid keys; missing={missing}, unexpected={extra}")
        self.value = value
        self.where = where

    def text(self, key: str, allowed: frozenset[str] | None = None) -> str:
        v = self.value[key]
        if not isinstance(v, str) or not v:
            raise ValueError(f"{self.where}.{key} must be a non-empty string")
        if allowed is not None and v not in allowed:
            raise ValueError(f"{self.where}.{key} must be one of {sorted(allowed)}")
        return v

    def integer(self, key: str) -> int:
        v = self.value[key]
        if not isinstance(v, int) or isinstance(v, bool):
            raise ValueError(f"{self.where}.{key} must be an integer")
        return v

    def boolean(self, key: str) -> bool:
        v = self.value[key]
        if not isinstance(v, bool):
            raise ValueError(f"{self.where}.{key} must be a boolean")
        return v

    def texts(self, key: str) -> tuple[str, ...]:
        v = self.value[key]
        if not isinstance(v, list) or not v:
            raise ValueError(f"{self.where}.{key} must be a non-empty array")
        if not all(isinstance(x, str) and x for x in v):
            raise ValueError(f"{self.where}.{key}[] must be non-empty strings")
        return tuple(v)

    def shape(self, key: str) -> tuple[int, int, int]:
        v = self.value[key]
        if not isinstance(v, list) or len(v) != 3:
            raise ValueError(f"{self.where}.{key} must contain three dimensions")
        if not all(isinstance(d, int) and not isinstance(d, bool) for d in v):
            raise ValueError(f"{self.where}.{key}[] must be integers")
        if min(v) < 1:
            raise ValueError(f"{self.where}.{key} dimensions must be positive")
        return (v[0], v[1], v[2])


def _case(value: object, index: int) -> GemmCase:
    r = _Reader(value, f"cases[{index}]", CASE_KEYS)
    priority = r.integer("priority")
    if priority not in (1, 2, 3):
        raise ValueError(f"cases[{index}].priority must be 1, 2, or 3")
    e = _Reader(r.value["evidence"], f"cases[{index}].evidence", frozenset({"kind", "note", "references"}))
    return GemmCase(
        id=r.text("id"), model=r.text("model"), workload=r.text("workload"),
        projection=r.text("projection"), shape=r.shape("shape"),
        input_output_dtype=r.text("input_output_dtype", DTYPE_NAMES),
        compute_dtype=r.text("compute_dtype", DTYPE_NAMES),
        weight_layout=r.text("weight_layout", frozenset({"out_in"})),
        bias=r.boolean("bias"), priority=priority,
        evidence=Evidence(e.text("kind", EVIDENCE_KINDS), e.text("note"), e.texts("references")),
    )


def load_corpus(path: Path = DEFAULT_CORPUS_PATH) -> GemmCorpus:
    top = _Reader(json.loads(Path(path).read_text()), "corpus",
                  frozenset({"schema_version", "name", "operator", "cases"}))
    version = top.integer("schema_version")
    if version != 1:
        raise ValueError(f"unsupported corpus schema version {version}")
    operator = top.text("operator")
    if operator != "torch.nn.functional.linear":
        raise ValueError(f"unsupported corpus operator {operator}")
    raw_cases = top.value["cases"]
    if not isinstance(raw_cases, list) or not raw_cases:
        raise ValueError("cases must be a non-empty array")
    cases = tuple(_case(c, i) for i, c in enumerate(raw_cases))
    if len({c.id for c in cases}) != len(cases):
        raise ValueError("case ids must be unique")
    return GemmCorpus(version, top.text("name"), operator, cases)
