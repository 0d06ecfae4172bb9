"""Run the per-case report harness over corpus cases, one process per case.

Same command line as the reference's ``benchmarks/run_corpus.py``
(chelokot/rdna3-fastmm, ``:11-134``): ``--list`` prints the cases;
``--case ID`` (repeatable) runs ``benchmark.py --operator linear --mode
dynamic --allow-unrecommended`` for each selected case into
``OUTPUT_DIRECTORY/<id>-<algorithm>.json``, each under its own timeout.
``--algorithm`` also accepts ``rank48`` here, since all three plans run on B200.
"""

from __future__ import annotations

import argparse
import subprocess
import sys
from dataclasses import dataclass
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from benchmarks.corpus import DEFAULT_CORPUS_PATH, GemmCase, load_corpus  # noqa: E402

BENCHMARK_SCRIPT = Path(__file__).resolve().parent / "benchmark.py"


@dataclass(frozen=True)
class RunnerConfig:
    algorithm: str
    output_directory: Path
    warmups: int
    rounds: int
    tile_size: int
    max_memory_fraction: float
    timeout_seconds: int
    allow_dirty: bool


def benchmark_command(case: GemmCase, config: RunnerConfig, output_path: Path) -> list[str]:
    command = [
        sys.executable, str(BENCHMARK_SCRIPT),
        "--algorithm", config.algorithm,
        "--operator", "linear",
        "--linear-implementation", "op",
        "--shape", ",".join(map(str, case.shape)),
        "--dtype", case.input_output_dtype,
        "--compute-dtype", case.compute_dtype,
        "--mode", "dynamic",
        "--warmups", str(config.warmups),
        "--rounds", str(config.rounds),
        "--tile-size", str(config.tile_size),
        "--max-memory-fraction", str(config.max_memory_fraction),
        "--allow-unrecommended",
        "--output", str(output_path),
    ]
    if not case.bias:
        command.append("--no-bias")
    if config.allow_dirty:
        command.append("--allow-dirty")
    return command


def parse_arguments(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--corpus", type=Path, default=DEFAULT_CORPUS_PATH)
    parser.add_argument("--algorithm", choices=("rank7", "rank48", "rank49"), default="rank49")
    selection = parser.add_mutually_exclusive_group(required=True)
    selection.add_argument("--list", action="store_true")
    selection.add_argument("--case", action="append")
    parser.add_argument("--output-directory", type=Path)
    parser.add_argument("--warmups", type=int, default=3)
    parser.add_argument("--rounds", type=int, default=9)
    parser.add_argument("--tile-size", type=int, default=8)
    parser.add_argument("--max-memory-fraction", type=float, default=0.30)
    parser.add_argument("--timeout-seconds", type=int, default=180)
    parser.add_argument("--allow-dirty", action="store_true")
    args = parser.parse_args(argv)
    if args.list:
        return args.corpus, None, None
    if args.output_directory is None:
        parser.error("--output-directory is required when running cases")
    if args.warmups < 1 or args.rounds < 3:
        parser.error("warmups must be positive and rounds must be at least three")
    if args.tile_size < 1 or args.timeout_seconds < 1:
        parser.error("tile size and timeout must be positive")
    if not 0 < args.max_memory_fraction <= 1:
        parser.error("max memory fraction must be in the interval (0, 1]")
    if len(args.case) != len(set(args.case)):
        parser.error("case ids must not be repeated")
    config = RunnerConfig(args.algorithm, args.output_directory, args.warmups, args.rounds,
                          args.tile_size, args.max_memory_fraction, args.timeout_seconds,
                          args.allow_dirty)
    return args.corpus, tuple(args.case), config


def format_case(case: GemmCase) -> str:
    shape = "x".join(map(str, case.shape))
    return f"{case.id}\tpriority={case.priority}\t{shape}\t{'bias' if case.bias else 'no-bias'}"


def main(argv=None) -> None:
    corpus_path, case_ids, config = parse_arguments(argv)
    corpus = load_corpus(corpus_path)
    if case_ids is None:
        for case in corpus.cases:
            print(format_case(case))
        return
    selected = [corpus.case(i) for i in case_ids]
    config.output_directory.mkdir(parents=True, exist_ok=True)
    for n, case in enumerate(selected, start=1):
        output = config.output_directory / f"{case.id}-{config.algorithm}.json"
        print(f"[{n}/{len(selected)}] {case.id} ({config.algorithm})", flush=True)
        subprocess.run(benchmark_command(case, config, output), check=True,
                       timeout=config.timeout_seconds)


if __name__ == "__main__":
    main()
