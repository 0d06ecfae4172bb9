"""Per-case benchmark report for the B200 backend (schema 2).

Same command line and report fields as the reference's harness
(``benchmarks/benchmark.py`` of chelokot/rdna3-fastmm: CLI ``:710-767``,
timing ``:127-157``, sampled correctness ``:160-265``, packing break-even
``:268-296``, memory estimate ``:299-319``, metrics ``:322-372``, report
``:375-707``), so B200 reports can be read next to the reference's RDNA3 ones:

    python rdna3-fastmm_b200/benchmarks/benchmark.py --algorithm rank7 \\
        --shape 4096,4096,12288 --operator linear --dtype bfloat16 \\
        --compute-dtype float16 --no-bias --mode dynamic --allow-unrecommended

Operations are timed one CUDA event pair each, in an order that rotates every
round; correctness compares a centred tile of every output macroblock with a
CPU FP32 product of the original inputs.  ``--linear-implementation op`` (the
reference's ``triton-op``) times the allocating ``torch.ops.rdna3_fastmm``
operator; ``plan`` times ``run_linear`` with a preallocated workspace.
``--sustained-seconds S`` (B200 addition) times each operation as a
back-to-back loop of about S seconds, the regime a power-capped GPU settles in.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import platform
import subprocess
import sys
import time
from dataclasses import asdict, dataclass
from datetime import UTC, datetime
from pathlib import Path
from statistics import median
from typing import Callable

import torch

PACKAGE_ROOT = Path(__file__).resolve().parent.parent
if str(PACKAGE_ROOT) not in sys.path:
    sys.path.insert(0, str(PACKAGE_ROOT))

from rdna3_fastmm import _native  # noqa: E402
from rdna3_fastmm.external_mm import rdna3_rank49_dynamic_v1_out  # noqa: E402
from rdna3_fastmm.linear import rdna3_linear, rdna3_rank7_linear, rdna3_rank48_linear  # noqa: E402
from rdna3_fastmm.runtime import (  # noqa: E402
    PackedRight, PackedWeight, Rank7Plan, Rank48Plan, Rank49Plan, Rank343Plan,
)
from rdna3_fastmm.schemes import CERTIFICATE_ROOT  # noqa: E402

GENERATED_HEADER = PACKAGE_ROOT / "csrc" / "generated" / "fmm_schemes.cuh"
ARTIFACTS = {
    "rank7": (CERTIFICATE_ROOT / "2x2x2_rank7_15add" / "certificate.json", Rank7Plan, rdna3_rank7_linear),
    "rank49": (CERTIFICATE_ROOT / "4x4x4_rank49_159add" / "certificate.json", Rank49Plan, rdna3_linear),
    "rank48": (CERTIFICATE_ROOT / "4x4x4_rank48_accurate" / "certificate.json", Rank48Plan,
               rdna3_rank48_linear),
    "rank343": (CERTIFICATE_ROOT / "8x8x8_rank343_1661add" / "certificate.json", Rank343Plan, None),
}
OPERATOR_NAMES = {"rank7": "rdna3_fastmm::linear_rank7", "rank49": "rdna3_fastmm::linear",
                  "rank48": "rdna3_fastmm::linear_rank48", "rank343": "(none)"}
DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}
ENVIRONMENT_KEYS = ("CUDA_VISIBLE_DEVICES", "CUBLAS_WORKSPACE_CONFIG", "NCCL_DEBUG",
                    "FMM_LEAF_GEMM_VARIANT", "FMM_RECONSTRUCT_VARIANT", "PYTORCH_CUDA_ALLOC_CONF")


@dataclass(frozen=True)
class TimingSummary:
    raw_ms: list
    median_ms: float
    first_quartile_ms: float
    third_quartile_ms: float


@dataclass(frozen=True)
class ErrorSummary:
    sample_count: int
    relative_l2_error: float
    maximum_absolute_error: float
    nonfinite_count: int


def parse_shape(text: str) -> tuple[int, int, int]:
    parts = tuple(int(p) for p in text.split(","))
    if len(parts) != 3 or min(parts) < 1:
        raise argparse.ArgumentTypeError("shape must contain three positive integers")
    return parts  # type: ignore[return-value]


def file_sha256(path: Path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def git(*args: str) -> str | None:
    """``git`` output, or None outside a git checkout (a copied source tree)."""
    try:
        result = subprocess.run(("git", *args), check=True, capture_output=True, text=True,
                                cwd=PACKAGE_ROOT)
    except (OSError, subprocess.CalledProcessError):
        return None
    return result.stdout.strip()


def tree_state() -> tuple[str | None, bool | None]:
    """(commit, dirty); both None when the tree is not a git checkout."""
    commit = git("rev-parse", "HEAD")
    if commit is None:
        return None, None
    return commit, bool(git("status", "--porcelain"))


def require_clean(dirty: bool | None, allow_dirty: bool) -> None:
    if dirty is None and not allow_dirty:
        raise RuntimeError("not a git checkout: the tree state is unknown; pass --allow-dirty")
    if dirty and not allow_dirty:
        raise RuntimeError("refusing to benchmark a dirty tree without --allow-dirty")


def quartile(values: list, which: int) -> float:
    """Linear-interpolated quartile (which = 1 or 3)."""
    ordered = sorted(values)
    pos = (len(ordered) - 1) * which / 4
    lo = int(pos)
    hi = min(lo + 1, len(ordered) - 1)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (pos - lo)


def summarize(values: list) -> TimingSummary:
    return TimingSummary(list(values), median(values), quartile(values, 1), quartile(values, 3))


def timed_ms(operation: Callable[[], None]) -> float:
    begin = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    begin.record()
    operation()
    end.record()
    end.synchronize()
    return float(begin.elapsed_time(end))


def loop_count(single_ms: float, sustained_seconds: float) -> int:
    """Calls in one sustained measurement: enough to last ``sustained_seconds``."""
    return max(1, round(sustained_seconds * 1e3 / max(single_ms, 1e-3)))


def measure_operations(operations: dict, warmups: int, rounds: int, sustained_seconds: float = 0.0):
    """Every operation once per round, the starting operation rotating.

    With ``sustained_seconds > 0`` each measurement is instead one event pair
    around a back-to-back loop lasting about that long, divided by the call
    count: on a power-capped part a single call is timed at whatever clock the
    previous operation left, while the loop reaches the steady clock that
    operation sustains on its own.
    """
    names = list(operations)

    def rotated(k: int) -> list:
        k %= len(names)
        return names[k:] + names[:k]

    for w in range(warmups):
        for name in rotated(w):
            operations[name]()
    torch.cuda.synchronize()
    counts = dict.fromkeys(names, 1)
    if sustained_seconds > 0:
        counts = {n: loop_count(timed_ms(operations[n]), sustained_seconds) for n in names}

    def measured(name: str) -> float:
        op, n = operations[name], counts[name]
        if n == 1:
            return timed_ms(op)

        def loop():
            for _ in range(n):
                op()
        return timed_ms(loop) / n

    raw = {name: [] for name in names}
    schedule = []
    for r in range(rounds):
        order = rotated(r)
        schedule.append(order)
        for name in order:
            raw[name].append(measured(name))
    return {name: summarize(v) for name, v in raw.items()}, schedule


def timing_method(sustained_seconds: float) -> str:
    if sustained_seconds > 0:
        return (f"one CUDA event pair around a back-to-back loop of about {sustained_seconds:g} s "
                "per operation, divided by the call count")
    return "one operation per CUDA event pair"


def macroblock_tile_starts(dimension: int, tile: int, scheme_size: int) -> list:
    """Start of a centred ``tile`` inside each of the ``scheme_size`` blocks."""
    block = -(-dimension // scheme_size)
    starts = []
    for b in range(scheme_size):
        lo, hi = b * block, min((b + 1) * block, dimension)
        if hi - lo < tile:
            raise ValueError("every macroblock must contain one sample tile")
        starts.append(lo + (hi - lo - tile) // 2)
    return starts


def validate_outputs(left, right, bias, outputs: dict, baseline: str, tile: int, scheme_size: int):
    rows = macroblock_tile_starts(left.shape[0], tile, scheme_size)
    cols = macroblock_tile_starts(right.shape[1], tile, scheme_size)
    left_slabs = [left.narrow(0, r, tile).float().cpu() for r in rows]
    right_slabs = [right.narrow(1, c, tile).float().cpu() for c in cols]
    sq_diff = dict.fromkeys(outputs, 0.0)
    max_abs = dict.fromkeys(outputs, 0.0)
    nonfinite = dict.fromkeys(outputs, 0)
    sq_ref = 0.0
    per_tile = []
    for i, r in enumerate(rows):
        for j, c in enumerate(cols):
            ref = left_slabs[i] @ right_slabs[j]
            if bias is not None:
                ref = ref + bias.narrow(0, c, tile).float().cpu()
            ref_sq = float(ref.double().square().sum())
            sq_ref += ref_sq
            entry = {}
            for name, out in outputs.items():
                cand = out.narrow(0, r, tile).narrow(1, c, tile).float().cpu()
                finite = torch.isfinite(cand)
                diff = torch.where(finite, cand - ref, torch.zeros_like(ref))
                d2 = float(diff.double().square().sum())
                m = float(diff.abs().max())
                nf = int((~finite).sum())
                sq_diff[name] += d2
                max_abs[name] = max(max_abs[name], m)
                nonfinite[name] += nf
                entry[name] = {"relative_l2_error": math.sqrt(d2 / ref_sq) if ref_sq else 0.0,
                               "maximum_absolute_error": m, "nonfinite_count": nf}
            per_tile.append({"macroblock": [i, j], "row_start": r, "column_start": c, "algorithms": entry})
    samples = len(rows) * len(cols) * tile * tile
    aggregate = {name: ErrorSummary(samples, math.sqrt(sq_diff[name] / sq_ref), max_abs[name], nonfinite[name])
                 for name in outputs}
    base = aggregate[baseline].relative_l2_error
    return {
        "aggregate": {n: asdict(s) for n, s in aggregate.items()},
        "candidate_to_baseline_error_ratio": {n: s.relative_l2_error / base if base else None
                                              for n, s in aggregate.items() if n != baseline},
        "per_tile": per_tile,
    }


def measure_packing(pack: Callable[[], object]):
    first = pack()
    torch.cuda.synchronize()
    del first
    torch.cuda.empty_cache()
    begin = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    wall = time.perf_counter()
    begin.record()
    packed = pack()
    end.record()
    end.synchronize()
    wall = time.perf_counter() - wall
    return packed, {"device_ms": float(begin.elapsed_time(end)), "wall_ms": wall * 1e3, "warmup_calls": 1}


def packing_break_even_reuses(packing_ms: float, reference_ms: float, prepacked_ms: float):
    """Calls after which packing has paid for itself (None if it never does)."""
    saved = reference_ms - prepacked_ms
    return math.ceil(packing_ms / saved) if saved > 0 else None


def memory_requirement_bytes(shape, plan, modes, has_bias: bool, keeps_replaced_output: bool = False) -> int:
    rows, inner, columns = shape
    elements = rows * inner + inner * columns + (1 + len(modes)) * rows * columns
    if keeps_replaced_output:
        elements += rows * columns
    workspace = 0
    if "dynamic" in modes or "external" in modes:
        workspace += plan.workspace_bytes * (("dynamic" in modes) + ("external" in modes))
    if "prepacked" in modes:
        workspace += plan.prepacked_workspace_bytes + plan.packed_right_bytes
    return (elements + (columns if has_bias else 0)) * plan.dtype.itemsize + workspace


def algorithm_metrics(timings: dict, shape, plan, operator: str, baseline: str, implementation: str):
    rows, inner, columns = shape
    classical = 2 * rows * inner * columns
    s = plan.shape
    leaf = 2 * plan.rank * s.block_rows * s.block_inner * s.block_columns
    kind = type(plan).__name__
    apis = {
        "torch_mm": "torch.mm(out=...)",
        "torch_linear": "torch.nn.functional.linear(input, weight, bias)",
        "candidate_dynamic": (f"{kind}.run(..., output=...)" if operator == "mm" else
                              f"{kind}.run_linear(...)" if implementation == "plan" else
                              f"{OPERATOR_NAMES[plan.scheme]} custom_op"),
        "candidate_prepacked": f"{kind}.run_linear_packed(...)" if operator == "linear" else
        f"{kind}.run_packed(..., output=...)",
        "candidate_external": "Inductor external_matmul out-callable",
    }
    base_ms = timings[baseline].median_ms
    metrics = {}
    for name, t in timings.items():
        entry = {"api": apis[name], "timing": asdict(t),
                 "effective_classical_tflops": classical / t.median_ms / 1e9}
        if name != baseline:
            entry["speedup"] = base_ms / t.median_ms
            entry["executed_leaf_tflops"] = leaf / t.median_ms / 1e9
        metrics[name] = entry
    return metrics


def benchmark(algorithm: str, shape, dtype, compute_dtype, modes, warmups: int, rounds: int,
              tile_size: int, seed: int, max_memory_fraction: float, allow_dirty: bool,
              allow_unrecommended: bool, operator: str = "mm", linear_bias: bool = True,
              linear_implementation: str = "op", sustained_seconds: float = 0.0) -> dict:
    commit, dirty = tree_state()
    require_clean(dirty, allow_dirty)
    if operator not in ("mm", "linear"):
        raise ValueError("operator must be mm or linear")
    if linear_implementation == "triton-op":
        linear_implementation = "op"
    if linear_implementation not in ("op", "plan"):
        raise ValueError("linear implementation must be op or plan")
    if operator == "linear" and any(m not in ("dynamic", "prepacked") for m in modes):
        raise ValueError("linear benchmarking supports dynamic and prepacked modes")
    if operator == "linear" and "prepacked" in modes and linear_implementation != "plan":
        raise ValueError("prepacked Linear benchmarking requires the plan implementation")
    if algorithm == "rank343" and operator != "mm":
        raise ValueError("rank 343 is a plain-mm (FP16) scheme")
    device = torch.device("cuda", torch.cuda.current_device())
    certificate, plan_type, operator_fn = ARTIFACTS[algorithm]
    plan = plan_type(*shape, device=device, dtype=dtype, compute_dtype=compute_dtype)
    if operator == "linear":
        recommended = {"dynamic": plan.is_linear_recommended(has_bias=linear_bias), "external": False,
                       "prepacked": plan.is_linear_recommended(has_bias=linear_bias, prepacked_weight=True)}
    else:
        recommended = {"dynamic": plan.is_recommended(),
                       "external": algorithm == "rank49" and dtype == torch.float16 and plan.is_recommended(),
                       "prepacked": plan.is_recommended(prepacked_right=True)}
    if not allow_unrecommended and not all(recommended[m] for m in modes):
        raise RuntimeError("shape or runtime is outside the measured dispatch whitelist")
    required = memory_requirement_bytes(shape, plan, modes, operator == "linear" and linear_bias,
                                        operator == "linear")
    free_before, _ = torch.cuda.mem_get_info(device)
    if required > free_before * max_memory_fraction:
        raise MemoryError(f"benchmark needs {required / 2**30:.2f} GiB, exceeding the "
                          f"{free_before * max_memory_fraction / 2**30:.2f} GiB budget")
    torch.manual_seed(seed)
    torch.cuda.manual_seed_all(seed)
    torch.cuda.reset_peak_memory_stats(device)
    rows, inner, columns = shape
    left = torch.randn((rows, inner), device=device, dtype=dtype)
    bias = None
    weight = None
    if operator == "linear":
        weight = torch.randn((columns, inner), device=device, dtype=dtype)
        right = weight.T
        bias = torch.randn((columns,), device=device, dtype=dtype) if linear_bias else None
        baseline = "torch_linear"
    else:
        right = torch.randn((inner, columns), device=device, dtype=dtype)
        baseline = "torch_mm"
    outputs = {baseline: torch.empty((rows, columns), device=device, dtype=dtype)}
    if operator == "linear":
        def run_baseline():
            outputs[baseline] = torch.nn.functional.linear(left, weight, bias)
    else:
        def run_baseline():
            torch.mm(left, right, out=outputs[baseline])
    operations = {baseline: run_baseline}
    packing = None
    if "dynamic" in modes:
        outputs["candidate_dynamic"] = torch.empty((rows, columns), device=device, dtype=dtype)
        ws = plan.allocate_workspace(1.0) if (operator == "mm" or linear_implementation == "plan") else None

        def run_dynamic():
            if operator == "linear":
                if linear_implementation == "op":
                    outputs["candidate_dynamic"] = operator_fn(left, weight, bias)
                else:
                    outputs["candidate_dynamic"] = plan.run_linear(left, weight, ws, bias,
                                                                   outputs["candidate_dynamic"])
            else:
                plan.run(left, right, ws, outputs["candidate_dynamic"])
        operations["candidate_dynamic"] = run_dynamic
    if "external" in modes:
        if algorithm != "rank49" or dtype != torch.float16:
            raise ValueError("the external_matmul candidate uses FP16 rank 49")
        outputs["candidate_external"] = torch.empty((rows, columns), device=device, dtype=dtype)
        operations["candidate_external"] = lambda: rdna3_rank49_dynamic_v1_out(
            left, right, out=outputs["candidate_external"])
    if "prepacked" in modes:
        outputs["candidate_prepacked"] = torch.empty((rows, columns), device=device, dtype=dtype)
        if operator == "linear":
            packed, packing = measure_packing(lambda: plan.pack_weight(weight, 1.0))
        else:
            packed, packing = measure_packing(lambda: plan.pack_right(right, 1.0))
        pws = plan.allocate_workspace(1.0, prepacked_right=True)

        def run_prepacked():
            if operator == "linear":
                assert isinstance(packed, PackedWeight)
                plan.run_linear_packed(left, packed, pws, bias, outputs["candidate_prepacked"])
            else:
                assert isinstance(packed, PackedRight)
                plan.run_packed(left, packed, pws, outputs["candidate_prepacked"])
        operations["candidate_prepacked"] = run_prepacked
    with torch.no_grad():
        timings, schedule = measure_operations(operations, warmups, rounds, sustained_seconds)
    torch.cuda.synchronize()
    correctness = validate_outputs(left, right, bias, outputs, baseline, tile_size, plan.scheme_size)
    algorithms = algorithm_metrics(timings, shape, plan, operator, baseline, linear_implementation)
    if packing is not None:
        pre = timings["candidate_prepacked"].median_ms
        if "candidate_dynamic" in timings:
            packing["break_even_reuses"] = packing_break_even_reuses(
                packing["device_ms"], timings["candidate_dynamic"].median_ms, pre)
            packing["break_even_reuses_vs_dynamic"] = packing["break_even_reuses"]
        packing["break_even_reuses_vs_baseline"] = packing_break_even_reuses(
            packing["device_ms"], timings[baseline].median_ms, pre)
        packing["first_call_ms"] = packing["device_ms"] + pre
    props = torch.cuda.get_device_properties(device)
    free_after, total = torch.cuda.mem_get_info(device)
    lib = _native.LIBRARY_PATH
    dname = str(dtype).removeprefix("torch.")
    cname = str(compute_dtype).removeprefix("torch.")
    return {
        "schema_version": 2,
        "generated_at_utc": datetime.now(UTC).isoformat(),
        "provenance": {
            "git_commit": commit,
            "git_dirty": dirty,
            "certificate_path": str(certificate.relative_to(PACKAGE_ROOT)),
            "certificate_sha256": file_sha256(certificate),
            "generated_module_path": str(GENERATED_HEADER.relative_to(PACKAGE_ROOT)),
            "generated_module_sha256": file_sha256(GENERATED_HEADER),
            "library_sha256": file_sha256(lib) if lib.exists() else None,
        },
        "runtime": {
            "python": platform.python_version(), "torch": torch.__version__, "cuda": torch.version.cuda,
            "library_version": _native.library().fmm_version(), "algorithm": plan.algorithm,
            "linear_implementation": linear_implementation if operator == "linear" else None,
            "input_output_dtype": dname, "compute_dtype": cname,
        },
        "device": {"name": props.name, "architecture": f"sm_{props.major}{props.minor}",
                   "multiprocessor_count": props.multi_processor_count, "total_memory_bytes": total},
        "environment": {k: os.environ.get(k) for k in ENVIRONMENT_KEYS},
        "protocol": {
            "seed": seed, "input_distribution": f"independent standard normal rounded to {dname}",
            "input_output_dtype": dname, "compute_dtype": cname, "warmup_rounds": warmups,
            "measured_rounds": rounds, "order_schedule": schedule,
            "timing_method": timing_method(sustained_seconds), "operator": operator,
            "weight_layout": "out_in" if operator == "linear" else "inner_columns",
            "bias": bias is not None,
            "correctness_reference": "CPU FP32 tile matmul from original inputs"
            + (" with FP32 bias addition" if bias is not None else ""),
            "tile_policy": f"centered {tile_size}x{tile_size} tile in each of "
            f"{plan.scheme_size ** 2} output macroblocks",
        },
        "case": {
            "shape": list(shape), "operator": operator, "recommended": recommended,
            "memory": {
                "estimated_required_bytes": required, "free_before_bytes": free_before,
                "free_after_bytes": free_after,
                "process_peak_allocated_bytes": torch.cuda.max_memory_allocated(device),
                "dynamic_workspace_bytes": plan.workspace_bytes,
                "prepacked_workspace_bytes": plan.prepacked_workspace_bytes,
                "packed_right_bytes": plan.packed_right_bytes,
                "packed_weight_bytes": plan.packed_weight_bytes,
            },
            "algorithms": algorithms, "packing": packing, "correctness": correctness,
        },
    }


def main(argv=None) -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--algorithm", choices=tuple(ARTIFACTS), required=True)
    parser.add_argument("--shape", type=parse_shape, required=True)
    parser.add_argument("--operator", choices=("mm", "linear"), default="mm")
    parser.add_argument("--linear-implementation", choices=("op", "triton-op", "plan"), default="op")
    parser.add_argument("--no-bias", action="store_true")
    parser.add_argument("--dtype", choices=tuple(DTYPES), default="float16")
    parser.add_argument("--compute-dtype", choices=tuple(DTYPES))
    parser.add_argument("--mode", choices=("dynamic", "prepacked", "external", "both"), default="both")
    parser.add_argument("--warmups", type=int, default=3)
    parser.add_argument("--rounds", type=int, default=9)
    parser.add_argument("--sustained-seconds", type=float, default=0.0,
                        help="time each operation as a back-to-back loop of about this long")
    parser.add_argument("--tile-size", type=int, default=16)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--max-memory-fraction", type=float, default=0.75)
    parser.add_argument("--allow-dirty", action="store_true")
    parser.add_argument("--allow-unrecommended", action="store_true")
    parser.add_argument("--output", type=Path)
    args = parser.parse_args(argv)
    if args.warmups < 1 or args.rounds < 3:
        parser.error("warmups must be positive and rounds must be at least three")
    if args.tile_size < 1:
        parser.error("tile size must be positive")
    if args.sustained_seconds < 0:
        parser.error("sustained seconds must not be negative")
    if args.no_bias and args.operator != "linear":
        parser.error("--no-bias requires --operator linear")
    if not 0 < args.max_memory_fraction <= 1:
        parser.error("max memory fraction must be in the interval (0, 1]")
    modes = ("dynamic", "prepacked") if args.mode == "both" else (args.mode,)
    dtype = DTYPES[args.dtype]
    compute = dtype if args.compute_dtype is None else DTYPES[args.compute_dtype]
    torch.set_grad_enabled(False)
    report = benchmark(args.algorithm, args.shape, dtype, compute, modes, args.warmups, args.rounds,
                       args.tile_size, args.seed, args.max_memory_fraction, args.allow_dirty,
                       args.allow_unrecommended, args.operator, not args.no_bias,
                       args.linear_implementation, args.sustained_seconds)
    text = json.dumps(report, indent=2, allow_nan=False) + "\n"
    if args.output is None:
        print(text, end="")
    else:
        args.output.write_text(text)
        print(args.output)


if __name__ == "__main__":
    main()
