"""Exact certificate checks (mirrors the reference's tests/test_slp.py:17-83,
tests/test_fastmm_certificate.py:10-44 and tests/test_verify_reduced_scheme.py:9-64)."""

import hashlib
import json
from copy import deepcopy
from fractions import Fraction

import pytest

from rdna3_fastmm import load_expanded_scheme
from rdna3_fastmm.certificate import load_reduced_scheme, verify_reduced_scheme
from rdna3_fastmm.schemes import CERTIFICATE_ROOT, get_scheme
from rdna3_fastmm.slp import load_and_verify_slp_certificate, load_slp_program

RANK48 = CERTIFICATE_ROOT / "4x4x4_rank48_accurate" / "certificate.json"
RANK49 = CERTIFICATE_ROOT / "4x4x4_rank49_159add" / "certificate.json"
RANK7 = CERTIFICATE_ROOT / "2x2x2_rank7_15add" / "certificate.json"
RANK343 = CERTIFICATE_ROOT / "8x8x8_rank343_1661add" / "certificate.json"


def test_rank48_slp_certificate_is_exact():
    certificate, summary = load_and_verify_slp_certificate(RANK48)
    assert summary.dimensions == (4, 4, 4)
    assert summary.rank == 48
    assert summary.additions == (80, 68, 108)
    assert summary.scalings == (4, 8, 16)
    assert summary.operations == (84, 76, 124)
    assert summary.tensor_entries == 64
    assert summary.sha256 == "c7103a1165af22d4e1a417607e9618b0bbae1b69e0c48ed7fa2a5aba26a3bcb7"
    assert tuple(len(p.assignments) for p in (certificate.left, certificate.right, certificate.output)) == (82, 60, 72)


@pytest.mark.parametrize("name,sha256", [
    ("left.slp", "af7719f288b346ae0dde8b8bf4a4a7bcf8d160ec8387c4a72d560a4bdb65f19b"),
    ("right.slp", "c09dda6d06633b9b438683819be49151c2ff24d26bca1097c8023ad534d390fa"),
    ("output.slp", "d441067f8e8d5d9c374ab2f290763ecc5f4738f989e1e3570d844d8207ed042f"),
])
def test_rank48_vendored_slp_matches_upstream(name, sha256):
    assert hashlib.sha256((RANK48.parent / name).read_bytes()).hexdigest() == sha256


@pytest.mark.parametrize("path,sha256", [
    (RANK7, "b374fcc797ea014994453b7502625e24f70ca2f1dcf1bdbe74a716342bfefb1e"),
    (RANK49, "a3c4121dfd09607045255628dd94b60133c24c46b65f1089e89c6564ba522561"),
    (RANK343, "c7afccb09f8491e484af1696c25c809757c4af649ee7220e79f25d1c7afe3955"),
])
def test_reduced_certificates_match_upstream(path, sha256):
    assert hashlib.sha256(path.read_bytes()).hexdigest() == sha256


def test_slp_rejects_unavailable_signal(tmp_path):
    path = tmp_path / "invalid.slp"
    path.write_text("o0:=i0+missing;\n")
    with pytest.raises(ValueError, match="unavailable signal missing"):
        load_slp_program(path, 1, 1)


def test_slp_rejects_nondyadic_scale(tmp_path):
    path = tmp_path / "invalid.slp"
    path.write_text("o0:=i0/3;\n")
    with pytest.raises(ValueError, match="dyadic"):
        load_slp_program(path, 1, 1)


def test_slp_rejects_missing_output(tmp_path):
    path = tmp_path / "invalid.slp"
    path.write_text("x0:=i0+i0;\n")
    with pytest.raises(ValueError, match=r"missing SLP outputs \[0\]"):
        load_slp_program(path, 1, 1)


def test_slp_rejects_unary_minus(tmp_path):
    path = tmp_path / "invalid.slp"
    path.write_text("o0:=-i0;\n")
    with pytest.raises(ValueError, match="unsupported SLP expression"):
        load_slp_program(path, 1, 1)


def test_load_expanded_rank_49_scheme():
    scheme = load_expanded_scheme(RANK49)
    assert scheme.dimensions == (4, 4, 4)
    assert scheme.rank == 49
    assert len(scheme.left_coefficients) == 49 and all(len(r) == 16 for r in scheme.left_coefficients)
    assert len(scheme.right_coefficients) == 49 and all(len(r) == 16 for r in scheme.right_coefficients)
    assert len(scheme.output_coefficients) == 16 and all(len(r) == 49 for r in scheme.output_coefficients)


def test_rank_49_certificate_is_exact():
    summary = verify_reduced_scheme(load_reduced_scheme(RANK49))
    assert summary.dimensions == (4, 4, 4)
    assert summary.rank == 49
    assert summary.side_additions == (42, 42, 75)
    assert summary.additions == 159
    assert summary.tensor_entries == 64


def test_rank_343_certificate_is_exact():
    summary = verify_reduced_scheme(load_reduced_scheme(RANK343))
    assert summary.dimensions == (8, 8, 8)
    assert (summary.rank, summary.additions, summary.side_additions) == (343, 1661, (462, 456, 743))
    assert summary.naive_additions == 4434


def test_rank343_program_reproduces_the_matrix_multiplication_tensor():
    """Integer check of the generator's rank-343 programs (numpy: 64^3 entries)."""
    import numpy as np

    scheme = get_scheme("rank343")
    U = np.array(scheme.left.coefficients(), dtype=np.int64)    # [343, 64]
    V = np.array(scheme.right.coefficients(), dtype=np.int64)   # [343, 64]
    W = np.array(scheme.output.coefficients(), dtype=np.int64)  # [64, 343]
    T = np.einsum("ri,rj,or->ijo", U, V, W)
    s = 8
    E = np.zeros_like(T)
    for row in range(s):
        for k in range(s):
            for col in range(s):
                E[row * s + k, k * s + col, row * s + col] = 1
    assert np.array_equal(T, E)
    assert scheme.certificate_sha256.startswith("c7afccb0")


def test_rank_7_certificate_is_exact():
    summary = verify_reduced_scheme(load_reduced_scheme(RANK7))
    assert (summary.rank, summary.additions, summary.side_additions) == (7, 15, (4, 4, 7))


def test_expanded_loader_rejects_invalid_brent_tensor(tmp_path):
    source = json.loads(RANK49.read_text())
    source["u"][0][0]["value"] *= -1
    path = tmp_path / "invalid-certificate.json"
    path.write_text(json.dumps(source))
    with pytest.raises(ValueError, match="Brent tensor"):
        load_expanded_scheme(path)


def _identity_panel():
    return {"n": [1, 1, 2], "m": 2, "z2": False, "complexity": {"naive": 0, "reduced": 0},
            "u_fresh": [], "v_fresh": [], "w_fresh": [],
            "u": [[{"index": 0, "value": 1}], [{"index": 0, "value": 1}]],
            "v": [[{"index": 0, "value": 1}], [{"index": 1, "value": 1}]],
            "w": [[{"index": 0, "value": 1}], [{"index": 1, "value": 1}]]}


def test_verify_reduced_scheme_accepts_exact_tensor():
    summary = verify_reduced_scheme(_identity_panel())
    assert (summary.dimensions, summary.rank, summary.additions, summary.tensor_entries) == ((1, 1, 2), 2, 0, 2)


@pytest.mark.parametrize("mutate,match", [
    (lambda s: s["w"].__setitem__(1, [{"index": 0, "value": 1}]), "Brent tensor"),
    (lambda s: s["complexity"].__setitem__("reduced", 1), "declared reduced"),
    (lambda s: s["u"].__setitem__(0, [{"index": 0, "value": 2}]), "non-signed"),
    (lambda s: s.__setitem__("z2", True), "non-Z2"),
    (lambda s: s.__setitem__("n", [0, 1, 2]), "positive integers"),
])
def test_verify_reduced_scheme_rejects(mutate, match):
    scheme = deepcopy(_identity_panel())
    mutate(scheme)
    with pytest.raises(ValueError, match=match):
        verify_reduced_scheme(scheme)


@pytest.mark.parametrize("name", ["rank7", "rank48", "rank49"])
def test_programs_reproduce_the_matrix_multiplication_tensor(name):
    """The linear programs the CUDA generator consumes encode the scheme
    exactly (row-major output blocks)."""
    scheme = get_scheme(name)
    s = scheme.size
    U, V, W = scheme.left.coefficients(), scheme.right.coefficients(), scheme.output.coefficients()
    total: dict = {}
    for r in range(scheme.rank):
        for i, a in enumerate(U[r]):
            for j, b in enumerate(V[r]):
                if a and b:
                    for o in range(s * s):
                        if W[o][r]:
                            total[(i, j, o)] = total.get((i, j, o), Fraction(0)) + a * b * W[o][r]
    total = {k: v for k, v in total.items() if v}
    expected = {(row * s + k, k * s + col, row * s + col): 1
                for row in range(s) for k in range(s) for col in range(s)}
    assert total == expected


def test_rank49_is_rank7_tensor_rank7():
    """Every rank-49 factor row is +-(rank-7 row (x) rank-7 row)."""
    r7, r49 = load_expanded_scheme(RANK7), load_expanded_scheme(RANK49)

    def kron_rows(rows):
        out = set()
        for a in rows:
            for b in rows:
                # block (i1, k1) of the outer level x (i2, k2) of the inner level
                v = []
                for i in range(4):
                    for k in range(4):
                        v.append(a[(i // 2) * 2 + k // 2] * b[(i % 2) * 2 + k % 2])
                out.add(tuple(v))
                out.add(tuple(-x for x in v))
        return out

    assert set(map(tuple, r49.left_coefficients)) <= kron_rows(r7.left_coefficients)
