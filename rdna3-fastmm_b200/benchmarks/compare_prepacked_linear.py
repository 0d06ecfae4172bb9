"""Rank 7 vs rank 49 vs rank 48, all prepacked, against native BF16 on one shape.

Same protocol and report as the reference's
``benchmarks/compare_prepacked_linear.py`` (chelokot/rdna3-fastmm, memory
estimate ``:68-100``, run ``:143-340``, CLI ``:343-382``): every plan packs the
one BF16 ``[N, K]`` weight (pack timed by ``measure_packing``), reuses its
workspace and output, and is timed with ``torch.mm(input, weight.T, out=...)``
in a rotating order; correctness samples a centred tile in each rank-48
output macroblock.  The status says whether rank 48 beats the faster of the
rank-7 and rank-49 controls; ``--require-rank48-win`` turns a loss into an
error.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import sys
from dataclasses import asdict, dataclass
from datetime import UTC, datetime
from pathlib import Path

import torch

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from benchmarks.benchmark import (  # noqa: E402
    ARTIFACTS, ENVIRONMENT_KEYS, GENERATED_HEADER, PACKAGE_ROOT, file_sha256, measure_operations,
    measure_packing, packing_break_even_reuses, parse_shape, require_clean, timing_method, tree_state,
    validate_outputs,
)
from rdna3_fastmm import _native  # noqa: E402
from rdna3_fastmm.runtime import Rank48Plan  # noqa: E402

PLAN_NAMES = ("rank7", "rank49", "rank48")
# cuBLAS workspace the native BF16 baseline may hold
LIBRARY_WORKSPACE_BYTES = 32 * 2**20


@dataclass(frozen=True)
class MemoryEstimate:
    source_bytes: int
    output_bytes: int
    plan_bytes: dict
    library_workspace_bytes: int
    total_bytes: int


def estimate_memory(shape, plans: dict) -> MemoryEstimate:
    rows, inner, columns = shape
    source = (rows * inner + columns * inner) * 2
    output = (len(plans) + 1) * rows * columns * 2
    per_plan = {n: p.prepacked_workspace_bytes + p.packed_weight_bytes for n, p in plans.items()}
    total = source + output + sum(per_plan.values()) + LIBRARY_WORKSPACE_BYTES
    return MemoryEstimate(source, output, per_plan, LIBRARY_WORKSPACE_BYTES, total)


def status(timings: dict) -> tuple[str, str, float]:
    """(status, fastest control, rank-48 speed-up over it)."""
    controls = {n: timings[n].median_ms for n in ("rank7", "rank49")}
    best = min(controls, key=controls.__getitem__)
    r48 = timings["rank48"].median_ms
    verdict = "rank48-wins" if r48 < controls[best] else "rank48-does-not-beat-current-control"
    return verdict, best, controls[best] / r48


def benchmark(shape, warmups: int, rounds: int, tile_size: int, seed: int, max_memory_fraction: float,
              allow_dirty: bool, allow_unrecommended: bool, sustained_seconds: float = 0.0) -> dict:
    commit, dirty = tree_state()
    require_clean(dirty, allow_dirty)
    device = torch.device("cuda", torch.cuda.current_device())
    plans = {n: ARTIFACTS[n][1](*shape, device=device, dtype=torch.bfloat16, compute_dtype=torch.float16)
             for n in PLAN_NAMES}
    if not allow_unrecommended and not plans["rank48"].is_linear_recommended(
            has_bias=False, prepacked_weight=True):
        raise RuntimeError("shape is outside the measured rank-48 prepacked gate")
    memory = estimate_memory(shape, plans)
    free_before, total = torch.cuda.mem_get_info(device)
    budget = int(free_before * max_memory_fraction)
    if memory.total_bytes > budget:
        raise MemoryError(f"benchmark needs {memory.total_bytes / 2**30:.2f} GiB, exceeding the "
                          f"{budget / 2**30:.2f} GiB budget")
    torch.manual_seed(seed)
    torch.cuda.manual_seed_all(seed)
    torch.cuda.reset_peak_memory_stats(device)
    rows, inner, columns = shape
    x = torch.randn((rows, inner), device=device, dtype=torch.bfloat16)
    weight = torch.randn((columns, inner), device=device, dtype=torch.bfloat16)
    outputs = {n: torch.empty((rows, columns), device=device, dtype=torch.bfloat16)
               for n in ("torch_bfloat16", *plans)}
    packed, packing = {}, {}
    for n, plan in plans.items():
        packed[n], timing = measure_packing(lambda plan=plan: plan.pack_weight(weight, 1.0))
        packing[n] = timing | {"packed_bytes": plan.packed_weight_bytes,
                               "weight_expansion": plan.packed_weight_bytes / (weight.numel() * 2)}
    workspaces = {n: p.allocate_workspace(1.0, prepacked_right=True) for n, p in plans.items()}
    operations = {"torch_bfloat16": lambda: torch.mm(x, weight.T, out=outputs["torch_bfloat16"])}
    for n, plan in plans.items():
        operations[n] = (lambda plan=plan, n=n: plan.run_linear_packed(
            x, packed[n], workspaces[n], output=outputs[n]))
    timings, order = measure_operations(operations, warmups, rounds, sustained_seconds)
    correctness = validate_outputs(x, weight.T, None, outputs, "torch_bfloat16", tile_size,
                                   Rank48Plan.scheme_size)
    native_ms = timings["torch_bfloat16"].median_ms
    verdict, best, r48_vs_best = status(timings)
    r48 = timings["rank48"].median_ms
    for n in plans:
        packing[n]["break_even_reuses_vs_native"] = packing_break_even_reuses(
            packing[n]["device_ms"], native_ms, timings[n].median_ms)
    props = torch.cuda.get_device_properties(device)
    free_after, _ = torch.cuda.mem_get_info(device)
    script = Path(__file__).resolve()
    return {
        "schema_version": 1,
        "status": verdict,
        "generated_at_utc": datetime.now(UTC).isoformat(),
        "provenance": {
            "git_commit": commit, "git_dirty": dirty,
            "benchmark_path": str(script.relative_to(PACKAGE_ROOT)),
            "benchmark_sha256": file_sha256(script),
            "artifacts": {n: {"certificate_path": str(ARTIFACTS[n][0].relative_to(PACKAGE_ROOT)),
                              "certificate_sha256": file_sha256(ARTIFACTS[n][0]),
                              "generated_module_path": str(GENERATED_HEADER.relative_to(PACKAGE_ROOT)),
                              "generated_module_sha256": file_sha256(GENERATED_HEADER)}
                          for n in PLAN_NAMES},
        },
        "runtime": {"python": platform.python_version(), "torch": torch.__version__,
                    "cuda": torch.version.cuda, "library_version": _native.library().fmm_version()},
        "device": {"name": props.name, "architecture": f"sm_{props.major}{props.minor}",
                   "multiprocessor_count": props.multi_processor_count, "total_memory_bytes": total},
        "environment": {k: os.environ.get(k) for k in ENVIRONMENT_KEYS},
        "protocol": {
            "shape": list(shape), "source_dtype": "bfloat16", "compute_dtype": "float16", "bias": False,
            "warmup_rounds": warmups, "measured_rounds": rounds, "order_schedule": order,
            "timing_method": timing_method(sustained_seconds),
            "allocation_contract": "all hot-path operations reuse output buffers; reduced-rank plans "
                                   "also reuse their prepacked weights and workspaces",
            "correctness_reference": "CPU FP32 tiles from original BF16 inputs",
            "tile_policy": f"centered {tile_size}x{tile_size} tile in each rank-48 output macroblock",
            "seed": seed,
        },
        "case": {
            "shape": list(shape),
            "timings": {n: asdict(t) for n, t in timings.items()},
            "speedup_vs_native": {n: native_ms / t.median_ms for n, t in timings.items()
                                  if n != "torch_bfloat16"},
            "rank48_speedup_vs_controls": {n: timings[n].median_ms / r48 for n in ("rank7", "rank49")},
            "best_current_control": best,
            "rank48_speedup_vs_best_current_control": r48_vs_best,
            "packing": packing,
            "correctness": correctness,
            "configs": {n: {"algorithm": p.algorithm,
                            "transform": asdict(p.transform_config(inner, columns)),
                            "weight_transform": asdict(p.weight_transform_config(inner, columns))}
                        for n, p in plans.items()},
            "memory": {"estimate": asdict(memory), "budget_bytes": budget, "free_before_bytes": free_before,
                       "free_after_bytes": free_after,
                       "process_peak_allocated_bytes": torch.cuda.max_memory_allocated(device)},
        },
    }


def main(argv=None) -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--shape", type=parse_shape, required=True)
    parser.add_argument("--warmups", type=int, default=1)
    parser.add_argument("--rounds", type=int, default=7)
    parser.add_argument("--sustained-seconds", type=float, default=0.0,
                        help="time each operation as a back-to-back loop of about this long")
    parser.add_argument("--tile-size", type=int, default=8)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--max-memory-fraction", type=float, default=0.5)
    parser.add_argument("--allow-dirty", action="store_true")
    parser.add_argument("--allow-unrecommended", action="store_true")
    parser.add_argument("--require-rank48-win", action="store_true")
    parser.add_argument("--output", type=Path)
    args = parser.parse_args(argv)
    if args.warmups < 1 or args.rounds < 3:
        parser.error("warmups must be positive and rounds must be at least three")
    if args.tile_size < 1:
        parser.error("tile size must be positive")
    if args.sustained_seconds < 0:
        parser.error("sustained seconds must not be negative")
    if not 0 < args.max_memory_fraction <= 1:
        parser.error("max memory fraction must be in the interval (0, 1]")
    torch.set_grad_enabled(False)
    report = benchmark(args.shape, args.warmups, args.rounds, args.tile_size, args.seed,
                       args.max_memory_fraction, args.allow_dirty, args.allow_unrecommended,
                       args.sustained_seconds)
    text = json.dumps(report, indent=2, allow_nan=False) + "\n"
    if args.output is None:
        print(text, end="")
    else:
        args.output.write_text(text)
        print(args.output)
    if args.require_rank48_win and report["status"] != "rank48-wins":
        raise RuntimeError("rank-48 did not beat the fastest current control")


if __name__ == "__main__":
    main()
