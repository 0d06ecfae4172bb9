"""The verified block schemes on the fast path, as linear programs.

Every scheme is loaded from its vendored certificate and verified exactly on
every load (integer Brent tensor for reduced circuits, Fraction Brent tensor
for the dyadic SLP).  The result is a :class:`Scheme` with three
:class:`~rdna3_fastmm.program.LinearProgram` s, all indexed row-major:

* ``left``  : input ``q`` = A block ``(q // s, q % s)``  -> left factor ``r``
* ``right`` : input ``q`` = B block ``(q // s, q % s)``  -> right factor ``r``
  (B = weight^T, so B block ``(kb, nb)`` is weight block ``(nb, kb)``)
* ``output``: input ``r`` = product ``r``  -> C block ``o = row * s + col``

Scheme identities (algorithm names, ranks, certificate digests) follow
``src/rdna3_fastmm/runtime.py:29-53, 780-880`` of chelokot/rdna3-fastmm.
Step order follows the reference schedulers
(``tools/generate_triton_scheme.py:27-67`` and
``tools/generate_slp_triton_scheme.py:15-62``), so the generated CUDA reads
in the same order as the reference kernels; the numerical result of every
signal depends only on its own expression tree.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path

from .certificate import load_reduced_scheme, verify_reduced_scheme
from .program import LinearProgram, Step, terms_to_expr
from .slp import load_and_verify_slp_certificate

CERTIFICATE_ROOT = Path(__file__).resolve().parent / "certificates"

__all__ = ["Scheme", "get_scheme", "SCHEME_NAMES", "SQUARE_SCHEME_NAMES", "CERTIFICATE_ROOT"]


@dataclass(frozen=True)
class Scheme:
    name: str
    algorithm: str
    scheme_id: int
    size: int
    rank: int
    certificate_sha256: str
    left: LinearProgram
    right: LinearProgram
    output: LinearProgram


def _schedule_circuit(
    inputs: int, gates: list, outputs: list, output_number: list[int]
) -> LinearProgram:
    """Gates in certificate order; each output as soon as its signals exist
    (lowest output first), as the reference generator schedules them."""
    steps: list[Step] = []
    pending = list(range(len(outputs)))
    available = inputs

    def flush() -> None:
        ready = [o for o in pending if all(t["index"] < available for t in outputs[o])]
        for o in ready:
            steps.append(Step("output", output_number[o], terms_to_expr(outputs[o])))
            pending.remove(o)

    flush()
    for g, terms in enumerate(gates):
        steps.append(Step("gate", g, terms_to_expr(terms)))
        available += 1
        flush()
    if pending:
        raise ValueError("output expressions reference unavailable signals")
    return LinearProgram(inputs, len(outputs), tuple(steps))


def _reduced_scheme(name: str, algorithm: str, folder: str) -> Scheme:
    path = CERTIFICATE_ROOT / folder / "certificate.json"
    source = load_reduced_scheme(path)
    summary = verify_reduced_scheme(source)
    n0, n1, n2 = summary.dimensions
    if not n0 == n1 == n2:
        raise ValueError("only square block schemes are supported")
    s, rank = n0, summary.rank
    left = _schedule_circuit(s * s, source["u_fresh"], source["u"], list(range(rank)))
    right = _schedule_circuit(s * s, source["v_fresh"], source["v"], list(range(rank)))
    # w outputs are column-major: output o is C block (o % s, o // s)
    row_major = [(o % s) * s + (o // s) for o in range(s * s)]
    output = _schedule_circuit(rank, source["w_fresh"], source["w"], row_major)
    digest = hashlib.sha256(path.read_bytes()).hexdigest()
    return Scheme(name, algorithm, rank, s, rank, digest, left, right, output)


def _slp_scheme(name: str, algorithm: str, folder: str) -> Scheme:
    certificate, summary = load_and_verify_slp_certificate(
        CERTIFICATE_ROOT / folder / "certificate.json"
    )
    n0, n1, n2 = summary.dimensions
    if not n0 == n1 == n2:
        raise ValueError("only square block schemes are supported")
    return Scheme(
        name,
        algorithm,
        summary.rank,
        n0,
        summary.rank,
        summary.sha256,
        certificate.left.to_linear_program(),
        certificate.right.to_linear_program(),
        certificate.output.to_linear_program(),
    )


SCHEME_NAMES = ("rank7", "rank48", "rank49")
# FP16 square plain-mm scheme (reference ``Rank343Plan``, ``runtime.py:883-962``)
SQUARE_SCHEME_NAMES = ("rank343",)

# pinned digests, as in the reference runtime's generated-module check
EXPECTED_SHA256 = {
    "rank7": "b374fcc797ea014994453b7502625e24f70ca2f1dcf1bdbe74a716342bfefb1e",
    "rank48": "c7103a1165af22d4e1a417607e9618b0bbae1b69e0c48ed7fa2a5aba26a3bcb7",
    "rank49": "a3c4121dfd09607045255628dd94b60133c24c46b65f1089e89c6564ba522561",
    "rank343": "c7afccb09f8491e484af1696c25c809757c4af649ee7220e79f25d1c7afe3955",
}


@lru_cache(maxsize=None)
def get_scheme(name: str) -> Scheme:
    if name == "rank7":
        scheme = _reduced_scheme("rank7", "rank7-v1", "2x2x2_rank7_15add")
    elif name == "rank49":
        scheme = _reduced_scheme("rank49", "rank49-v1", "4x4x4_rank49_159add")
    elif name == "rank48":
        scheme = _slp_scheme("rank48", "rank48-accurate-v1", "4x4x4_rank48_accurate")
    elif name == "rank343":
        scheme = _reduced_scheme("rank343", "rank343-mfma-v1", "8x8x8_rank343_1661add")
    else:
        raise ValueError(f"unknown scheme {name!r}")
    if scheme.certificate_sha256 != EXPECTED_SHA256[name]:
        raise RuntimeError(f"{name} certificate digest does not match the pinned value")
    return scheme
