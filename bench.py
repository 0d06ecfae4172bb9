"""Benchmark of the reduced-rank BF16 linear on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c3|c4|c5a|c5b]
                    [--impl native|reference]

A *step* is one ``F.linear`` of the workload through the B200 path: left
transform, weight transform (dynamic plans), tcgen05 leaf GEMM, reconstruct.
Each kernel is bracketed by CUDA events on the launching (current) stream, so
the line carries per-kernel-class times and roofline fractions; L2 is flushed
(a 256 MiB write) before every timed step, outside the events.

``value`` is effective TFLOP/s = 2*M*N*K / t summed over ranks (weak scaling:
every rank runs the whole workload on its own GPU; the path has no exchange
step).  ``e2e`` is the same metric through the public plan API with pinned
host buffers, host->device copies of A and the weight and the device->host
copy of C inside the timed region; consecutive steps alternate over two
streams with their own buffers, so one step's input copies overlap the
previous step's compute and result copy.  ``cpu_baseline`` is the CPU oracle on a
bounded row sample of the same workload.  ``--impl reference`` times that CPU
implementation alone (the reference is a ROCm/Triton project with no B200
path; its algorithm's CPU restatement is the reference arm).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "rdna3-fastmm_b200", ROOT / "tests" / "golden"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

WORKLOADS = {
    # name: (scheme, M, K, N, bias, prepacked, description)
    "c2": ("rank7", 4096, 4096, 12288, False, False,
           "rank-7 dynamic F.linear, DiT MLP-up: A[4096,4096] W[12288,4096], no bias"),
    "c3": ("rank7", 4992, 16384, 4096, True, False,
           "rank-7 dynamic F.linear + bias, MLP-down: A[4992,16384] W[4096,16384]"),
    "c4": ("rank49", 8214, 12288, 4608, False, True,
           "rank-49 prepacked: A[8214,12288] W[4608,12288], M%4 != 0"),
    "c5a": ("rank48", 8192, 8192, 8192, False, True, "rank-48 prepacked 8192^3"),
    "c5b": ("rank48", 65536, 4608, 12288, False, True,
            "rank-48 prepacked A[65536,4608] W[12288,4608]"),
}

MEASURED_PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> tuple[dict, str]:
    if MEASURED_PEAKS.exists():
        return json.loads(MEASURED_PEAKS.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(workload: str) -> float | None:
    """DRAM bytes per leaf-GEMM launch from the committed ncu summary."""
    path = ROOT / "profiles" / f"leaf_gemm_{workload}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip())
    return None


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """Poll NVML (read-only) every ~2 ms while the timed region runs: SM
    clock, max SM clock and the active clock-event (throttle) reasons."""

    REASONS = {  # NVML clocks-event-reason bits
        0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
        0x4: "sw_power_cap",
    }

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def poll():
                while not self._stop.is_set():
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM),
                                         reasons(handle)))
                    time.sleep(0.002)

            self._thread = threading.Thread(target=poll, daemon=True)
            self._thread.start()
        except Exception as error:  # NVML missing: report no samples
            self.error = repr(error)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        clocks = [c for c, _ in self.samples]
        reasons = set()
        for _, mask in self.samples:
            for bit, name in self.REASONS.items():
                if mask & bit:
                    reasons.add(name)
        out = {"sm_mhz": statistics.median(clocks) if clocks else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(reasons), "samples": len(clocks), "source": "nvml"}
        if self.error:
            out["error"] = self.error
        return out


# ---------------------------------------------------------------------- CPU arm
def cpu_sample(workload: str, target_seconds: float = 12.0) -> dict:
    """Time the CPU oracle (numpy, all host threads) on the workload.

    The weight transform runs once on the full weight (skipped for prepacked
    workloads, whose packing is outside a step); the per-row stages (left
    transform, leaf products, reconstruct) run on a row sample that is grown
    until it takes about a quarter of ``target_seconds`` and are scaled to M.
    """
    import numpy as np

    from inputs import f32, make_linear_inputs
    from oracle import fmm_oracle as oracle

    scheme, M, K, N, with_bias, prepacked, _ = WORKLOADS[workload]
    s = 4 if scheme != "rank7" else 2
    A_full, W, bias = make_linear_inputs(min(M, 64 * s), K, N, seed=0, bias=with_bias)
    w = f32(W)
    b = f32(bias) if bias is not None else None
    t0 = time.perf_counter()
    R = oracle.weight_transform(scheme, w)
    t_weight = 0.0 if prepacked else time.perf_counter() - t0
    R32 = R.astype(np.float32)

    def run(rows: int) -> float:
        A, _, _ = make_linear_inputs(rows, K, N, seed=0)
        a = f32(A)
        t = time.perf_counter()
        L = oracle.left_transform(scheme, a)
        P = np.matmul(L.astype(np.float32), R32).astype(np.float16)
        oracle.output_transform(scheme, P, rows, N, b)
        return time.perf_counter() - t

    rows = 64 * s
    elapsed = run(rows)
    while elapsed < target_seconds / 4 and rows * 2 <= M:
        rows *= 2
        elapsed = run(rows)
    total = t_weight + elapsed * (M / rows)
    flops = 2.0 * M * K * N
    return {"value": flops / total / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": (f"{scheme} CPU oracle (numpy, FP32 BLAS leaf products): weight transform "
                       f"{'excluded (prepacked)' if prepacked else f'{t_weight:.2f} s on the full weight'}"
                       f" + {rows} of {M} rows in {elapsed:.2f} s scaled to M; est. {total:.2f} s/step"),
            "seconds": total, "rows": rows}


# ---------------------------------------------------------------------- GPU arm
def run_native(args, rank: int, world: int, device) -> dict | None:
    import torch
    import torch.distributed as dist

    from inputs import make_linear_inputs
    from rdna3_fastmm import _native
    from rdna3_fastmm.runtime import Rank7Plan, Rank48Plan, Rank49Plan

    plans = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
    scheme, M_total, K, N, with_bias, prepacked, description = WORKLOADS[args.workload]
    if args.rows:
        M_total = args.rows
        description += f" (rows overridden to {M_total})"
    shard = args.shard and world > 1
    if shard:
        if M_total % (world * args.chunks):
            raise SystemExit("--shard needs M divisible by gpus * chunks")
        M = M_total // world
        if args.transport == "p2p":
            description += (f"; rows sharded block-cyclically over {world} GPUs in {args.chunks} chunks, "
                            f"output gathered by the reconstruct kernel itself (stores into every "
                            f"rank's peer-mapped buffer over NVLink), overlapped with compute")
        else:
            description += (f"; rows sharded block-cyclically over {world} GPUs in {args.chunks} chunks, "
                            f"output all-gathered (NCCL) chunk by chunk, overlapped with compute")
    else:
        M = M_total
    plan = plans[scheme](M, K, N, device, dtype=torch.bfloat16, compute_dtype=torch.float16)
    # every rank draws its own rows (seeded by rank), the weight is replicated
    A_h, W_h, b_h = make_linear_inputs(M, K, N, seed=0, bias=with_bias)
    if shard and rank:
        A_h = make_linear_inputs(M, K, 1, seed=100 + rank)[0]
    A, W = A_h.to(device), W_h.to(device)
    bias = b_h.to(device) if b_h is not None else None
    ws = plan.allocate_workspace(0.9, prepacked_right=prepacked)
    packed = plan.pack_weight(W, 0.9) if prepacked else None
    right = packed.transformed if prepacked else ws.right_transformed
    out = torch.empty((M, N), device=device, dtype=torch.bfloat16)
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)
    s = plan.shape
    stream = torch.cuda.current_stream(device)

    def step(ev):
        # the same launches as fmm_linear: prepacked -> left transform; dynamic ->
        # left and weight transform paired in one launch
        ev[0].record(stream)
        if prepacked:
            _native.transform_a(scheme, A, ws.left_transformed)
        else:
            _native.transform_aw(scheme, A, ws.left_transformed, W, right)
        ev[1].record(stream)
        ev[2].record(stream)
        _native.leaf_gemm(plan.rank, ws.left_transformed, right, s.block_rows, s.block_columns,
                          s.block_inner, ws.products)
        ev[3].record(stream)
        _native.reconstruct(scheme, ws.products, M, N, bias, out)
        ev[4].record(stream)
        ev[5].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        flush.zero_()
        step([torch.cuda.Event(enable_timing=True) for _ in range(6)])
    torch.cuda.synchronize(device)
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(device.index) as clocks:
        for ev in events:
            flush.zero_()
            step(ev)
        torch.cuda.synchronize(device)
        barrier()
    stages = {"transform_a": [], "transform_w": [], "leaf_gemm": [], "reconstruct": [], "all_gather": []}
    totals = []
    for ev in events:
        stages["transform_a"].append(ev[0].elapsed_time(ev[1]))
        stages["transform_w"].append(ev[1].elapsed_time(ev[2]))
        stages["leaf_gemm"].append(ev[2].elapsed_time(ev[3]))
        stages["reconstruct"].append(ev[3].elapsed_time(ev[4]))
        stages["all_gather"].append(ev[4].elapsed_time(ev[5]))
        totals.append(ev[0].elapsed_time(ev[5]))
    total_ms = sum(totals)
    if shard:
        from rdna3_fastmm.distributed import RowShardedLinear

        p2p = args.transport == "p2p"
        layer = RowShardedLinear(plans[scheme], M_total, W, bias=bias, chunks=args.chunks,
                                 reserve_sms=args.reserve_sms,
                                 max_free_memory_fraction=0.9, transport=args.transport)
        gathered = None if p2p else layer.gather_buffer()
        for _ in range(args.warmup):
            flush.zero_()
            layer(A, out=gathered)
        torch.cuda.synchronize(device)
        barrier()
        shard_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                        for _ in range(args.steps)]
        with ClockSampler(device.index) as shard_clocks:
            for e0, e1 in shard_events:
                flush.zero_()
                e0.record(stream)
                layer(A, out=gathered)
                e1.record(stream)
            torch.cuda.synchronize(device)
            barrier()
        compute_ms = total_ms
        total_ms = sum(a.elapsed_time(b) for a, b in shard_events)
        clocks = shard_clocks
    status, _ = _native.device_status(device.index)
    if status:
        raise RuntimeError(f"device status {status:#x} after the timed region")
    if args.profile:
        if rank == 0:
            _emit({"profile_run": args.workload, "M": M, "K": K, "N": N,
                   "ms_per_step": total_ms / args.steps,
                   "stages_ms": {k: statistics.mean(v) for k, v in stages.items()}})
        return None

    # parity spot check of this very output against the FP64 product (sampled rows)
    rows = torch.arange(0, M, max(1, M // 64), device=device)
    exact = A[rows].double() @ W.double().T
    if bias is not None:
        exact += bias.double()
    got = out[rows].double()
    rel = float(torch.linalg.vector_norm(got - exact) / torch.linalg.vector_norm(exact))
    native_rows = torch.nn.functional.linear(A[rows], W, bias).double()
    native_rel = float(torch.linalg.vector_norm(native_rows - exact) / torch.linalg.vector_norm(exact))
    nonfinite = int((~torch.isfinite(out)).sum())  # over the whole output

    # cuBLAS BF16 on the same GPU and inputs (context, not the product)
    for _ in range(3):
        torch.nn.functional.linear(A, W, bias)
    cub = []
    for _ in range(max(5, min(args.steps, 20))):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        torch.nn.functional.linear(A, W, bias, )
        e1.record(stream)
        cub.append((e0, e1))
    torch.cuda.synchronize(device)
    cublas_ms = statistics.median(a.elapsed_time(b) for a, b in cub)

    # End to end through the public plan API with pinned host buffers.  Steps
    # alternate over `lanes` streams, each with its own device inputs,
    # workspace, output and pinned result buffer, so the host->device copies of
    # step k+1 run while step k computes and copies its result back (PCIe is
    # full duplex); every step still copies all of its inputs in and its whole
    # result out inside the timed region.
    A_pin, W_pin = A_h.pin_memory(), W_h.pin_memory()
    b_pin = b_h.pin_memory() if b_h is not None else None
    lanes = 1 if shard else max(1, args.e2e_lanes)
    lane_state = []
    for k in range(lanes):
        lane = {"stream": stream if lanes == 1 else torch.cuda.Stream(device=device),
                "A": torch.empty_like(A), "W": torch.empty_like(W),
                "b": torch.empty_like(bias) if bias is not None else None}
        if shard:
            lane["C_pin"] = torch.empty((layer.rows if gathered is None else gathered.shape[0], N),
                                        dtype=torch.bfloat16).pin_memory()
        else:
            lane["ws"] = ws if k == 0 else plan.allocate_workspace(0.9, prepacked_right=prepacked)
            lane["out"] = out if k == 0 else torch.empty_like(out)
            lane["C_pin"] = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
        lane_state.append(lane)

    def e2e_step(lane):
        with torch.cuda.stream(lane["stream"]):
            A_d, W_d, b_d = lane["A"], lane["W"], lane["b"]
            A_d.copy_(A_pin, non_blocking=True)
            if not prepacked:
                W_d.copy_(W_pin, non_blocking=True)
            if b_d is not None:
                b_d.copy_(b_pin, non_blocking=True)
            if shard:
                res = layer(A_d, out=gathered)
            elif prepacked:
                res = plan.run_linear_packed(A_d, packed, lane["ws"], b_d, lane["out"])
            else:
                res = plan.run_linear(A_d, W_d, lane["ws"], b_d, lane["out"])
            lane["C_pin"].copy_(res, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 10))
    e2e_steps += (-e2e_steps) % lanes
    for k in range(2 * lanes):
        e2e_step(lane_state[k % lanes])
    torch.cuda.synchronize(device)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for lane in lane_state:
        lane["stream"].wait_event(e0)
    for k in range(e2e_steps):
        e2e_step(lane_state[k % lanes])
    for lane in lane_state:
        stream.wait_stream(lane["stream"])
    e1.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    C_pin = lane_state[0]["C_pin"]
    h2d = A_h.numel() * 2 + (0 if prepacked else W_h.numel() * 2) + (N * 2 if b_h is not None else 0)
    d2h = C_pin.numel() * 2

    local = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = float(local[0]), float(local[1])
    if shard:
        layer.close()  # collective: unmaps the peers' gather buffers (p2p)
    if rank != 0:
        return None

    flops = 2.0 * M * N * K  # this rank's share
    job_flops = 2.0 * M_total * N * K if shard else world * flops
    ms_per_step = total_ms / args.steps
    pk, pk_kind = peaks()
    leaf_flops = 2.0 * plan.rank * s.block_rows * s.block_inner * s.block_columns
    gemm_ms = statistics.mean(stages["leaf_gemm"])
    achieved = leaf_flops / (gemm_ms * 1e-3) / 1e12
    # the burst peak while the timed region ran at full clock, the sustained
    # (power-capped) peak when the clock record shows the cap or a lower clock
    clock = clocks.summary()
    capped = "sw_power_cap" in clock["reasons"] or (
        clock["sm_mhz"] is not None and clock["sm_max_mhz"] and clock["sm_mhz"] < 0.95 * clock["sm_max_mhz"])
    peak_name = "bf16_tflops_sustained" if capped and "bf16_tflops_sustained" in pk else "bf16_tflops"
    peak = pk[peak_name]
    a_bytes = M * K * 2 + plan.rank * s.block_rows * s.block_inner * 2
    w_bytes = N * K * 2 + plan.rank * s.block_columns * s.block_inner * 2
    r_bytes = plan.rank * s.block_rows * s.block_columns * 2 + M * N * 2 + (N * 2 if with_bias else 0)
    gemm_bytes = plan.rank * (s.block_rows + s.block_columns) * s.block_inner * 2 \
        + plan.rank * s.block_rows * s.block_columns * 2

    def hbm(nbytes, ms):
        if ms <= 0:
            return None
        gbs = nbytes / (ms * 1e-3) / 1e9
        return {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 3),
                "bytes": nbytes}

    kernels = {
        "transform_a": hbm(a_bytes, statistics.mean(stages["transform_a"])) if prepacked else None,
        "transforms_aw": None if prepacked else hbm(a_bytes + w_bytes, statistics.mean(stages["transform_a"])),
        "leaf_gemm": {"ms": round(gemm_ms, 4), "tflops": round(achieved, 1),
                      "frac": round(achieved / peak, 3), "flops": leaf_flops},
        "reconstruct": hbm(r_bytes, statistics.mean(stages["reconstruct"])),
    }
    if shard:
        moved = (world - 1) * M * N * 2  # bytes each rank receives
        kernels["sharded_step"] = {"ms": round(ms_per_step, 4), "compute_only_ms": round(compute_ms / args.steps, 4),
                                   "gather_bytes_received": moved, "chunks": args.chunks,
                                   "nvlink_gbs_if_gather_bound": round(moved / (ms_per_step * 1e-3) / 1e9, 1)}
    traffic = profile_traffic(args.workload)
    line = {
        "metric": "effective TFLOP/s (2MNK/t) per B200 and at 8 GPUs; speedup vs cuBLAS BF16",
        "value": round(job_flops / (ms_per_step * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if shard else "weak",
        "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 leaves, fp32 accumulate",
        "data": "synthetic (seeded A~N(0,1), W~N(0,0.02) BF16)",
        "config": {"workload": f"{args.workload}: {description}", "scheme": scheme,
                   "M": M, "K": K, "N": N, "bias": with_bias, "prepacked": prepacked,
                   "l2": "flushed (256 MiB write) before every step",
                   "parallelism": (f"rows sharded x{world} + "
                                   + ("fused reconstruct/all-gather over NVLink peer memory"
                                      if args.transport == "p2p" else "NCCL all-gather") if shard else
                                   f"replicas x{world}" if world > 1 else "single GPU")},
        "roofline": {"bound": "tensor", "kernel": "leaf_gemm", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 3),
                     "peak_source": f"{pk_kind} {peak_name} (dense FP16 == BF16 rate; "
                                    f"{'power-capped' if capped else 'full-clock'} timed region)",
                     "traffic": traffic, "algorithmic_bytes": gemm_bytes},
        "kernels": kernels,
        "cublas_bf16": {"ms": round(cublas_ms, 4),
                        "tflops": round(flops / (cublas_ms * 1e-3) / 1e12, 1),
                        "speedup": round(cublas_ms / ms_per_step, 3)},
        "accuracy": {"rel_l2_vs_fp64": rel, "native_bf16_rel_l2": native_rel,
                     "ratio": rel / native_rel if native_rel else None, "sampled_rows": int(rows.numel()),
                     "nonfinite_outputs": nonfinite},
        "e2e": {"value": round(job_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": ("RowShardedLinear (gather)" if shard else
                f"{type(plan).__name__}.run_linear{'_packed' if prepacked else ''}"),
                "streams": lanes},
        "clocks": clocks.summary(),
        "gpu_launches": args.steps * 3,
    }
    return line


def _emit(line: dict) -> None:
    os.write(_JSON_FD, (json.dumps(line) + "\n").encode())


_JSON_FD = 1


def main() -> None:
    global _JSON_FD
    # libraries (NCCL's version banner, for one) may write to stdout; keep
    # the real stdout for the single JSON line and send everything else to stderr
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=100)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    parser.add_argument("--impl", default="native", choices=["native", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--rows", type=int, default=0,
                        help="override M (smaller cases for profiler captures)")
    parser.add_argument("--shard", action="store_true",
                        help="split M over the ranks and all-gather C (strong scaling)")
    parser.add_argument("--e2e-lanes", type=int, default=2,
                        help="streams the e2e steps alternate over, each with its own buffers, so "
                             "one step's host->device copies overlap the previous step's compute "
                             "and device->host copy (1: strictly one step after another)")
    parser.add_argument("--chunks", type=int, default=None,
                        help="row chunks per rank in --shard mode (default: 4 with the NCCL gather, "
                             "which overlaps the next chunk; 1 with --transport p2p, whose gathering "
                             "reconstruct is already NVLink-bound)")
    parser.add_argument("--reserve-sms", type=int, default=32,
                        help="SMs the GEMM leaves free, while --shard chunks compute, for the NCCL "
                             "all-gather or the gathering reconstruct of the previous chunk")
    parser.add_argument("--transport", choices=("nccl", "p2p"), default="nccl",
                        help="--shard gather: NCCL all-gather, or the reconstruct kernel storing "
                             "into every rank's peer-mapped buffer over NVLink")
    parser.add_argument("--profile", action="store_true",
                        help="timed steps only: no cuBLAS, e2e, parity or CPU legs")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.chunks is None:
        args.chunks = 1 if args.transport == "p2p" else 4

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        # each step is one bounded sample (a few seconds); at most 5 are taken so
        # that the arm ends within a couple of minutes whatever --steps is
        samples = [cpu_sample(args.workload, target_seconds=4.0) for _ in range(min(args.steps, 5))]
        value = statistics.median(s["value"] for s in samples)
        base = dict(samples[0])
        base["value"] = value
        _emit({
            "impl": "reference",
            "metric": "effective TFLOP/s (2MNK/t) per B200 and at 8 GPUs; speedup vs cuBLAS BF16",
            "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 in/out, fp16 leaves", "data": "synthetic",
            "config": {"workload": f"{args.workload}: {WORKLOADS[args.workload][6]}"},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        })
        return

    import torch
    import torch.distributed as dist

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    try:
        line = run_native(args, rank, world, device)
        if line is not None and rank == 0:
            if not args.no_cpu_baseline:
                cpu = cpu_sample(args.workload)
                line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
            _emit(line)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
