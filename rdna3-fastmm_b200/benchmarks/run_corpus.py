"""Run the per-case report harness (``benchmark.py``) over corpus cases.

Command line (flag names and output file names as in the reference's
``benchmarks/run_corpus.py``, so scripts written for it run unchanged):

    run_corpus.py --list [--corpus FILE]
    run_corpus.py --case ID [--case ID ...] --output-directory DIR
                  [--algorithm rank7|rank48|rank49] [--warmups W] [--rounds R]
                  [--tile-size T] [--max-memory-fraction F] [--timeout-seconds S]
                  [--allow-dirty]

Each selected case runs as its own ``benchmark.py --operator linear --mode
dynamic --allow-unrecommended`` process (a fresh CUDA context per case, so
one case's allocations or a crash cannot affect the next) writing
``DIR/<id>-<algorithm>.json``.  Unlike a fail-fast loop, every case runs even
when an earlier one fails or times out; ``DIR/run-<algorithm>.json`` records
each case's outcome and duration, and the exit status is non-zero when any
case did not finish cleanly.  ``--algorithm rank48`` is accepted because all
three plans run on B200.
"""

from __future__ import annotations

import argparse
import json
import subprocess
import sys
import time
from dataclasses import asdict, dataclass
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from benchmarks.corpus import DEFAULT_CORPUS_PATH, GemmCase, load_corpus  # noqa: E402

BENCHMARK_SCRIPT = Path(__file__).resolve().parent / "benchmark.py"
ALGORITHMS = ("rank7", "rank48", "rank49")


@dataclass(frozen=True)
class RunnerConfig:
    """Settings shared by every case of one corpus run."""

    algorithm: str
    output_directory: Path
    warmups: int
    rounds: int
    tile_size: int
    max_memory_fraction: float
    timeout_seconds: int
    allow_dirty: bool

    def problems(self) -> list[str]:
        """Why these settings cannot run (empty when they can)."""
        found = []
        if self.algorithm not in ALGORITHMS:
            found.append(f"--algorithm must be one of {', '.join(ALGORITHMS)}")
        if self.warmups < 1:
            found.append("--warmups needs at least one untimed call")
        if self.rounds < 3:
            found.append("--rounds needs at least three timed calls for quartiles")
        if self.tile_size < 1:
            found.append("--tile-size must be at least 1")
        if self.timeout_seconds < 1:
            found.append("--timeout-seconds must be at least 1")
        if not 0.0 < self.max_memory_fraction <= 1.0:
            found.append("--max-memory-fraction lies outside (0, 1]")
        return found

    def output_for(self, case: GemmCase) -> Path:
        return self.output_directory / f"{case.id}-{self.algorithm}.json"


def benchmark_command(case: GemmCase, config: RunnerConfig, output_path: Path) -> list[str]:
    """The ``benchmark.py`` invocation that measures one case as a dynamic linear."""
    options = {
        "--algorithm": config.algorithm,
        "--operator": "linear",
        "--linear-implementation": "op",
        "--shape": "{},{},{}".format(*case.shape),
        "--dtype": case.input_output_dtype,
        "--compute-dtype": case.compute_dtype,
        "--mode": "dynamic",
        "--warmups": config.warmups,
        "--rounds": config.rounds,
        "--tile-size": config.tile_size,
        "--max-memory-fraction": config.max_memory_fraction,
        "--output": output_path,
    }
    switches = ["--allow-unrecommended"]
    switches += [] if case.bias else ["--no-bias"]
    switches += ["--allow-dirty"] if config.allow_dirty else []
    command = [sys.executable, str(BENCHMARK_SCRIPT)]
    for flag, value in options.items():
        command += [flag, str(value)]
    return command + switches


def _parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--corpus", type=Path, default=DEFAULT_CORPUS_PATH)
    parser.add_argument("--algorithm", default="rank49")
    what = parser.add_mutually_exclusive_group(required=True)
    what.add_argument("--list", action="store_true", help="print the corpus cases and exit")
    what.add_argument("--case", action="append", metavar="ID", help="case id to run (repeatable)")
    parser.add_argument("--output-directory", type=Path)
    parser.add_argument("--warmups", type=int, default=3)
    parser.add_argument("--rounds", type=int, default=9)
    parser.add_argument("--tile-size", type=int, default=8)
    parser.add_argument("--max-memory-fraction", type=float, default=0.30)
    parser.add_argument("--timeout-seconds", type=int, default=180)
    parser.add_argument("--allow-dirty", action="store_true")
    return parser


def parse_arguments(argv=None):
    """``(corpus path, case ids or None, RunnerConfig or None)``; ``None`` ids
    mean ``--list``.  Invalid settings exit through argparse with every
    problem listed at once."""
    parser = _parser()
    args = parser.parse_args(argv)
    if args.list:
        return args.corpus, None, None
    problems = []
    if args.output_directory is None:
        problems.append("--output-directory is required when running cases")
    repeated = sorted({c for c in args.case if args.case.count(c) > 1})
    if repeated:
        problems.append(f"case ids given more than once: {', '.join(repeated)}")
    config = RunnerConfig(args.algorithm, args.output_directory or Path("."), args.warmups, args.rounds,
                          args.tile_size, args.max_memory_fraction, args.timeout_seconds, args.allow_dirty)
    problems += config.problems()
    if problems:
        parser.error("; ".join(problems))
    return args.corpus, tuple(args.case), config


def format_case(case: GemmCase) -> str:
    """One ``--list`` line: id, priority, MxKxN, bias."""
    return "\t".join((case.id, f"priority={case.priority}", "x".join(str(d) for d in case.shape),
                      "bias" if case.bias else "no-bias"))


@dataclass
class CaseOutcome:
    case: str
    output: str
    status: str  # "ok", "failed", "timeout"
    returncode: int | None
    seconds: float


def run_case(case: GemmCase, config: RunnerConfig) -> CaseOutcome:
    output = config.output_for(case)
    started = time.monotonic()
    try:
        done = subprocess.run(benchmark_command(case, config, output), timeout=config.timeout_seconds)
        status, code = ("ok" if done.returncode == 0 else "failed"), done.returncode
    except subprocess.TimeoutExpired:
        status, code = "timeout", None
    return CaseOutcome(case.id, str(output), status, code, round(time.monotonic() - started, 3))


def main(argv=None) -> int:
    corpus_path, case_ids, config = parse_arguments(argv)
    corpus = load_corpus(corpus_path)
    if case_ids is None:
        print("\n".join(format_case(case) for case in corpus.cases))
        return 0
    cases = [corpus.case(case_id) for case_id in case_ids]  # unknown ids fail before any run
    config.output_directory.mkdir(parents=True, exist_ok=True)
    outcomes = []
    for position, case in enumerate(cases, start=1):
        print(f"[{position}/{len(cases)}] {case.id} ({config.algorithm})", flush=True)
        outcomes.append(run_case(case, config))
        if outcomes[-1].status != "ok":
            print(f"  {case.id}: {outcomes[-1].status}", file=sys.stderr, flush=True)
    record = {"corpus": str(corpus_path), "config": {k: str(v) for k, v in asdict(config).items()},
              "cases": [asdict(o) for o in outcomes]}
    (config.output_directory / f"run-{config.algorithm}.json").write_text(json.dumps(record, indent=2) + "\n")
    return 0 if all(o.status == "ok" for o in outcomes) else 1


if __name__ == "__main__":
    sys.exit(main())
