"""Build ``rdna3_fastmm/_lib/libfmm_sm100.so`` in-tree with nvcc (sm_100a).

    python rdna3-fastmm_b200/build.py [--verbose]

One translation unit (``csrc/fmm_api.cu``) holds every kernel; the CUDA
runtime is linked statically so the library loads on a host without a GPU
(the driver is only needed when a kernel is launched).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCE = HERE / "csrc" / "fmm_api.cu"
OUTPUT = HERE / "rdna3_fastmm" / "_lib" / "libfmm_sm100.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-shared", "-cudart", "static",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found")
    return found


def sources() -> list[Path]:
    return [SOURCE, *sorted((HERE / "csrc").rglob("*.cuh")), ROOT / "include" / "fmm_sm100.h"]


def up_to_date() -> bool:
    if not OUTPUT.exists():
        return False
    built = OUTPUT.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in sources())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and up_to_date():
        return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-I", str(HERE / "csrc"),
           str(SOURCE), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(verbose=args.verbose, force=args.force))
    sys.exit(0)
