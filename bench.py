"""Benchmark of the reduced-rank BF16 linear on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c3|c4|c4r49|c5a|c5b]
                    [--impl native|reference] [--replicas] [--transport nccl|p2p|ce]

Default workload: c5b, ``A[65536,4608] x W[12288,4608]^T`` through the rank-48
prepacked plan -- the largest configuration of the benchmark set that fits one
B200 (10.8 GB of planes).  A *step* is one ``F.linear`` of the workload through
the B200 path: left transform (plus the weight transform for dynamic
workloads), tcgen05 leaf GEMM, reconstruct.  Each kernel is bracketed by CUDA
events on the launching (current) stream, so the line carries per-kernel-class
times and roofline fractions; L2 is flushed (a 256 MiB write) before every
timed step, outside the events.

One GPU: ``value`` is effective TFLOP/s = 2*M*N*K / t.

N GPUs (``torchrun``): the rows of ``A`` are sharded evenly over the ranks,
the packed weight is replicated (packed on every rank), and every rank runs
its rows through the same three launches (strong scaling: the job's work is
fixed).  Two numbers are measured, both as the max over ranks of CUDA-event
time:

* ``value``: the whole ``C[M, N]`` gathered on every rank
  (``RowShardedLinear``; by default the transport measured fastest at that
  GPU count: at 2 GPUs ``ce`` -- each finished row chunk copied into the peer's
  buffer by the copy engines while the next chunk computes -- and from 3 GPUs
  up ``p2p`` -- the reconstruct kernel stores every rank's rows into all
  peers' buffers over NVLink; ``--transport nccl``: NCCL all-gather of
  finished row chunks overlapped with the next chunk);
* ``no_gather``: each rank keeps its own rows (the caller does not need the
  gathered output), no data-path collective.

``--replicas`` instead runs one full copy of the workload per GPU (weak
scaling).  ``e2e`` is the same metric through the public API with pinned host
buffers (bound to the GPU's NUMA node): host->device copies of the step's
inputs and the device->host copy of the step's result inside the timed region
(sharded: each rank copies in its rows of ``A`` and copies out its own rows of
the result).  ``accuracy`` is the error gate against an FP64 product on
centred macroblock tiles (``rdna3_fastmm.accuracy``), on the gathered output
when sharded.  ``cpu_baseline`` is the CPU oracle on a bounded row sample of
the same workload.  ``--impl reference`` times that CPU implementation alone
(the reference is a ROCm/Triton project with no B200 path; its algorithm's
CPU restatement is the reference arm).
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
    # c4 names rank 49; with FP16 leaves rank 49 misses the 1.2x error gate
    # (~1.7x native BF16), so the shape runs on rank 48 -- the plan the
    # reference itself measured best for 8214x12288x4608.  c4r49 keeps rank 49.
    "c4": ("rank48", 8214, 12288, 4608, False, True,
           "A[8214,12288] W[4608,12288] prepacked, M%4 != 0; rank 48 in place of rank 49 "
           "(rank 49 fails the 1.2x error gate with FP16 leaves)"),
    "c4r49": ("rank49", 8214, 12288, 4608, False, True,
              "rank-49 prepacked: A[8214,12288] W[4608,12288], M%4 != 0 (fails the 1.2x error gate)"),
    "c5a": ("rank48", 8192, 8192, 8192, False, True, "rank-48 prepacked 8192^3"),
    "c5b": ("rank48", 65536, 4608, 12288, False, True,
            "rank-48 prepacked A[65536,4608] W[12288,4608]"),
}
DEFAULT_WORKLOAD = "c5b"

METRIC = "effective TFLOP/s (2MNK/t) per B200 and at 8 GPUs; speedup vs cuBLAS BF16"
MEASURED_PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> tuple[dict, str]:
    if MEASURED_PEAKS.exists():
        return json.loads(MEASURED_PEAKS.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(workload: str) -> tuple[float | None, str | None]:
    """DRAM bytes per leaf-GEMM launch from the committed ncu summary."""
    path = ROOT / "profiles" / f"leaf_gemm_{workload}.md"
    if not path.exists():
        return None, None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip()), f"profiles/{path.name}"
    return None, None


# ---------------------------------------------------------------------- host placement
def bind_to_gpu_numa(index: int) -> set | None:
    """Restrict this process to the CPUs NVML reports as local to GPU
    ``index`` (so pinned host buffers, allocated afterwards, sit on the GPU's
    NUMA node).  Returns the previous affinity, or None when nothing changed."""
    try:
        import pynvml

        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(index)
        words = (os.cpu_count() + 63) // 64
        mask = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
        cpus = {64 * w + b for w, word in enumerate(mask) for b in range(64) if (word >> b) & 1}
        previous = os.sched_getaffinity(0)
        cpus &= previous
        if not cpus or cpus == previous:
            return None
        os.sched_setaffinity(0, cpus)
        return previous
    except Exception:
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
        self.power_mw: list[int] = []
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
                    try:
                        self.power_mw.append(pynvml.nvmlDeviceGetPowerUsage(handle))
                    except Exception:  # power readings unsupported: clocks only
                        pass
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
               "sm_mhz_min": min(clocks) if clocks else None,
               "reasons": sorted(reasons), "samples": len(clocks), "source": "nvml"}
        if self.power_mw:
            out["power_w_median"] = round(statistics.median(self.power_mw) / 1000, 1)
            out["power_w_max"] = round(max(self.power_mw) / 1000, 1)
        if self.error:
            out["error"] = self.error
        return out


# ---------------------------------------------------------------------- CPU arm
_WEIGHT_PLANES: dict = {}


def cpu_sample(workload: str, target_seconds: float = 12.0) -> dict:
    """Time the CPU oracle (numpy, all host threads) on the workload.

    The weight transform runs on the full weight (timed only for dynamic
    workloads; a prepacked workload transforms its weight once, outside a
    step, and the planes are reused between samples); the per-row stages
    (left transform, leaf products, reconstruct) run on a row sample that is
    grown until it takes about a quarter of ``target_seconds`` and are scaled
    to M.
    """
    import numpy as np

    from inputs import f32, make_linear_inputs
    from oracle import fmm_oracle as oracle

    scheme, M, K, N, with_bias, prepacked, _ = WORKLOADS[workload]
    s = 4 if scheme != "rank7" else 2
    _, W, bias = make_linear_inputs(s, K, N, seed=0, bias=with_bias)
    b = f32(bias) if bias is not None else None
    t0 = time.perf_counter()
    if prepacked and workload in _WEIGHT_PLANES:
        R32 = _WEIGHT_PLANES[workload]
    else:
        R32 = oracle.weight_transform(scheme, f32(W)).astype(np.float32)
        if prepacked:
            _WEIGHT_PLANES[workload] = R32
    t_weight = 0.0 if prepacked else time.perf_counter() - t0

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
    return {"value": flops / total / 1e12, "unit": "TFLOP/s", "cores": len(os.sched_getaffinity(0)),
            "kind": "port",
            "sample": (f"{scheme} CPU oracle (numpy, FP32 BLAS leaf products): weight transform "
                       f"{'excluded (prepacked)' if prepacked else f'{t_weight:.2f} s on the full weight'}"
                       f" + {rows} of {M} rows in {elapsed:.2f} s scaled to M; est. {total:.2f} s/step"),
            "seconds": total, "rows": rows}


# ---------------------------------------------------------------------- GPU arm
def _events(n: int):
    import torch

    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


class StagedStep:
    """One step of the workload as its three launches, each between CUDA
    events on the current stream: the input-side transform(s), the leaf GEMM,
    the reconstruct."""

    def __init__(self, plan, scheme: str, prepacked: bool, A, W, bias, workspace, right, out):
        self.plan, self.scheme, self.prepacked = plan, scheme, prepacked
        self.A, self.W, self.bias, self.ws, self.right, self.out = A, W, bias, workspace, right, out

    def __call__(self, ev, stream) -> None:
        from rdna3_fastmm import _native

        s, ws = self.plan.shape, self.ws
        ev[0].record(stream)
        if self.prepacked:
            _native.transform_a(self.scheme, self.A, ws.left_transformed)
        else:
            _native.transform_aw(self.scheme, self.A, ws.left_transformed, self.W, self.right)
        ev[1].record(stream)
        _native.leaf_gemm(self.plan.rank, ws.left_transformed, self.right, s.block_rows, s.block_columns,
                          s.block_inner, ws.products)
        ev[2].record(stream)
        _native.reconstruct(self.scheme, ws.products, s.rows, s.columns, self.bias, self.out)
        ev[3].record(stream)


def timed(run, steps: int, warmup: int, flush, stream, device, barrier, n_events: int = 2):
    """Warm up, then time ``steps`` calls of ``run(events, stream)`` with a
    barrier and a synchronize on both sides; NVML clocks sampled meanwhile.
    L2 is flushed before every call, outside the events."""
    import torch

    for _ in range(warmup):
        flush.zero_()
        run(_events(n_events), stream)
    torch.cuda.synchronize(device)
    events = [_events(n_events) for _ in range(steps)]
    barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(device.index) as clocks:
        for ev in events:
            flush.zero_()
            run(ev, stream)
        torch.cuda.synchronize(device)
        barrier()
    return events, clocks.summary()


def stage_times(events) -> dict:
    names = ("transform", "leaf_gemm", "reconstruct")
    out = {n: [ev[i].elapsed_time(ev[i + 1]) for ev in events] for i, n in enumerate(names)}
    out["step"] = [ev[0].elapsed_time(ev[3]) for ev in events]
    return out


def cublas_ms(A, W, bias, flush, stream, device, repeats: int) -> float:
    import torch

    for _ in range(3):
        torch.nn.functional.linear(A, W, bias)
    pairs = []
    for _ in range(repeats):
        flush.zero_()
        e0, e1 = _events(2)
        e0.record(stream)
        torch.nn.functional.linear(A, W, bias)
        e1.record(stream)
        pairs.append((e0, e1))
    torch.cuda.synchronize(device)
    return statistics.median(a.elapsed_time(b) for a, b in pairs)


def kernel_report(plan, M: int, N: int, K: int, with_bias: bool, prepacked: bool, stages: dict,
                  clock: dict) -> tuple[dict, dict, float]:
    """Per-kernel-class times and roofline fractions of one rank's step."""
    pk, pk_kind = peaks()
    s = plan.shape
    leaf_flops = 2.0 * plan.rank * s.block_rows * s.block_inner * s.block_columns
    gemm_ms = statistics.mean(stages["leaf_gemm"])
    achieved = leaf_flops / (gemm_ms * 1e-3) / 1e12
    # the burst peak while the timed region ran at full clock, the sustained
    # (power-capped) peak when the clock record shows the cap or a lower clock
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
        gbs = nbytes / (ms * 1e-3) / 1e9
        return {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 3),
                "bytes": nbytes, "of": f"{pk_kind} hbm_gbs {pk['hbm_gbs']}"}

    t_ms = statistics.mean(stages["transform"])
    kernels = {
        "transform_a": hbm(a_bytes, t_ms) if prepacked else None,
        "transforms_aw": None if prepacked else hbm(a_bytes + w_bytes, t_ms),
        "leaf_gemm": {"ms": round(gemm_ms, 4), "tflops": round(achieved, 1),
                      "frac": round(achieved / peak, 3), "flops": leaf_flops,
                      "of": f"{pk_kind} {peak_name} {peak}"},
        "reconstruct": hbm(r_bytes, statistics.mean(stages["reconstruct"])),
    }
    roofline = {"bound": "tensor", "kernel": "leaf_gemm", "achieved": round(achieved, 1),
                "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 3),
                "peak_source": f"{pk_kind} {peak_name} (dense FP16 == BF16 rate; "
                               f"{'power-capped' if capped else 'full-clock'} timed region)",
                "algorithmic_bytes": gemm_bytes}
    return kernels, roofline, gemm_ms


def pinned(shape, dtype):
    import torch

    return torch.empty(shape, dtype=dtype).pin_memory()


def e2e_single(plan, prepacked: bool, packed, A_h, W_h, b_h, ws, out, lanes: int, steps: int,
               stream, device):
    """The plan API end to end: each step copies its inputs in from pinned host
    memory and its whole result out.  Consecutive steps alternate over `lanes`
    streams, each with its own device inputs, workspace, output and pinned
    result buffer, so step k+1's host->device copies overlap step k's compute
    and result copy (PCIe is full duplex)."""
    import torch

    A_pin, W_pin = A_h.pin_memory(), W_h.pin_memory()
    b_pin = b_h.pin_memory() if b_h is not None else None
    M, N = out.shape
    lane_state = []
    for k in range(lanes):
        lane_state.append({
            "stream": stream if lanes == 1 else torch.cuda.Stream(device=device),
            "A": torch.empty(A_h.shape, dtype=A_h.dtype, device=device),
            "W": None if prepacked else torch.empty(W_h.shape, dtype=W_h.dtype, device=device),
            "b": torch.empty(b_h.shape, dtype=b_h.dtype, device=device) if b_h is not None else None,
            "ws": ws if k == 0 else plan.allocate_workspace(0.9, prepacked_right=prepacked),
            "out": out if k == 0 else torch.empty_like(out),
            "C_pin": pinned((M, N), torch.bfloat16),
        })

    def step(lane):
        with torch.cuda.stream(lane["stream"]):
            lane["A"].copy_(A_pin, non_blocking=True)
            if not prepacked:
                lane["W"].copy_(W_pin, non_blocking=True)
            if lane["b"] is not None:
                lane["b"].copy_(b_pin, non_blocking=True)
            if prepacked:
                res = plan.run_linear_packed(lane["A"], packed, lane["ws"], lane["b"], lane["out"])
            else:
                res = plan.run_linear(lane["A"], lane["W"], lane["ws"], lane["b"], lane["out"])
            lane["C_pin"].copy_(res, non_blocking=True)

    n = steps + (-steps) % lanes
    for k in range(2 * lanes):
        step(lane_state[k % lanes])
    torch.cuda.synchronize(device)
    e0, e1 = _events(2)
    e0.record(stream)
    for lane in lane_state:
        lane["stream"].wait_event(e0)
    for k in range(n):
        step(lane_state[k % lanes])
    for lane in lane_state:
        stream.wait_stream(lane["stream"])
    e1.record(stream)
    torch.cuda.synchronize(device)
    h2d = A_h.numel() * 2 + (0 if prepacked else W_h.numel() * 2) + (b_h.numel() * 2 if b_h is not None else 0)
    return e0.elapsed_time(e1) / n, h2d, M * N * 2, n * 3


def run_native(args, rank: int, world: int, device) -> dict | None:
    import torch
    import torch.distributed as dist

    from inputs import make_linear_inputs
    from rdna3_fastmm import _native
    from rdna3_fastmm.accuracy import error_gate
    from rdna3_fastmm.runtime import Rank7Plan, Rank48Plan, Rank49Plan

    plans = {"rank7": Rank7Plan, "rank48": Rank48Plan, "rank49": Rank49Plan}
    scheme, M_total, K, N, with_bias, prepacked, description = WORKLOADS[args.workload]
    if args.rows:
        M_total = args.rows
        description += f" (rows overridden to {M_total})"
    plan_type = plans[scheme]
    shard = world > 1 and not args.replicas
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(*values: float) -> list[float]:
        t = torch.tensor(values, dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t]

    if shard:
        if M_total % (world * args.chunks):
            raise SystemExit("sharding needs M divisible by gpus * chunks")
        M = M_total // world
        # one global input: every rank holds the same A and takes its rows
        A_full, W_h, b_h = make_linear_inputs(M_total, K, N, seed=0, bias=with_bias)
        A_h = A_full[rank * M:(rank + 1) * M].contiguous()
    else:
        M = M_total
        A_full = None
        A_h, W_h, b_h = make_linear_inputs(M, K, N, seed=0, bias=with_bias)

    # ---- this rank's rows through the three launches (per-kernel events)
    plan = plan_type(M, K, N, device, dtype=torch.bfloat16, compute_dtype=torch.float16)
    A, W = A_h.to(device), W_h.to(device)
    bias = b_h.to(device) if b_h is not None else None
    ws = plan.allocate_workspace(0.9, prepacked_right=prepacked)
    packed = plan.pack_weight(W, 0.9) if prepacked else None
    right = packed.transformed if prepacked else ws.right_transformed
    out = torch.empty((M, N), device=device, dtype=torch.bfloat16)
    staged = StagedStep(plan, scheme, prepacked, A, W, bias, ws, right, out)
    events, clock = timed(staged, args.steps, args.warmup, flush, stream, device, barrier, n_events=4)
    stages = stage_times(events)
    local_ms = sum(stages["step"])
    launches = args.steps * 3

    gathered_line = None
    if shard:
        from rdna3_fastmm.distributed import RowShardedLinear

        p2p = args.transport in ("p2p", "ce")  # the layer gathers into its own peer-mapped buffer
        layer = RowShardedLinear(plan_type, M_total, W, bias=bias, chunks=args.chunks,
                                 reserve_sms=args.reserve_sms, max_free_memory_fraction=0.9,
                                 transport=args.transport)
        local_rows = layer.local_rows(A_full).to(device)
        gather_out = None if p2p else layer.gather_buffer()

        def gathered_step(ev, strm):
            ev[0].record(strm)
            layer(local_rows, out=gather_out)
            ev[1].record(strm)

        g_events, g_clock = timed(gathered_step, args.steps, args.warmup, flush, stream, device, barrier)
        gathered_ms_total = sum(a.elapsed_time(b) for a, b in g_events)
        launches += args.steps * 3 * args.chunks
        gathered_line = {"ms_total": gathered_ms_total, "clock": g_clock}

    status, _ = _native.device_status(device.index)
    if status:
        raise RuntimeError(f"device status {status:#x} after the timed region")
    if args.profile:
        if rank == 0:
            _emit({"profile_run": args.workload, "M": M, "K": K, "N": N,
                   "ms_per_step": local_ms / args.steps,
                   "stages_ms": {k: statistics.mean(v) for k, v in stages.items()}})
        return None

    # ---- the error gate on this run's output (the gathered one when sharded)
    accuracy = None
    if shard:
        result = layer(local_rows, out=gather_out)
        torch.cuda.synchronize(device)
        barrier()
        if rank == 0:
            accuracy = error_gate(A_full, W, bias, result, plan.scheme_size)
            accuracy["on"] = f"gathered C[{M_total},{N}] on rank 0 (rows from all {world} ranks)"
        torch.cuda.synchronize(device)
        barrier()
    else:
        accuracy = error_gate(A, W, bias, out, plan.scheme_size)
        accuracy["on"] = f"C[{M},{N}] of the last timed step"

    cub_ms = cublas_ms(A, W, bias, flush, stream, device, max(5, min(args.steps, 20)))

    # ---- end to end through the public API, pinned host buffers
    prev_affinity = None if args.no_numa_bind else bind_to_gpu_numa(device.index)
    if shard:
        # each rank copies its rows in and its own rows of the gathered result out
        rows_pin = layer.local_rows(A_full).pin_memory()
        rows_dev = torch.empty_like(local_rows)
        blocks = layer.row_blocks()
        own_pin = pinned((layer.count, N), torch.bfloat16)

        def e2e_step():
            rows_dev.copy_(rows_pin, non_blocking=True)
            res = layer(rows_dev, out=gather_out)
            at = 0
            for start, count in blocks:
                own_pin[at:at + count].copy_(res[start:start + count], non_blocking=True)
                at += count

        e2e_n = max(3, min(args.steps, 10))
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(device)
        barrier()
        e0, e1 = _events(2)
        e0.record(stream)
        for _ in range(e2e_n):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / e2e_n
        h2d, d2h = rows_pin.numel() * 2, own_pin.numel() * 2
        launches += e2e_n * 3 * args.chunks
        e2e_api, lanes = f"RowShardedLinear ({args.transport} gather)", 1
    else:
        lanes = max(1, args.e2e_lanes)
        e2e_ms, h2d, d2h, e2e_launches = e2e_single(plan, prepacked, packed, A_h, W_h, b_h, ws, out, lanes,
                                                    max(3, min(args.steps, 10)), stream, device)
        launches += e2e_launches
        e2e_api = f"{type(plan).__name__}.run_linear{'_packed' if prepacked else ''}"
    if prev_affinity is not None:
        os.sched_setaffinity(0, prev_affinity)

    g_total = gathered_line["ms_total"] if shard else 0.0
    local_ms, e2e_ms, g_total = max_over_ranks(local_ms, e2e_ms, g_total)
    if shard:
        layer.close()  # collective: unmaps the peers' gather buffers (p2p)
    if rank != 0:
        return None

    flops_rank = 2.0 * M * N * K  # one rank's share
    job_flops = 2.0 * M_total * N * K if shard else world * flops_rank
    local_step_ms = local_ms / args.steps
    kernels, roofline, _ = kernel_report(plan, M, N, K, with_bias, prepacked, stages, clock)
    traffic, traffic_src = profile_traffic(args.workload) if not shard and not args.rows else (None, None)
    roofline["traffic"] = traffic
    if traffic_src:
        roofline["traffic_source"] = traffic_src
    pk, pk_kind = peaks()
    line = {
        "metric": METRIC,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 leaves, fp32 accumulate",
        "data": "synthetic (seeded A~N(0,1), W~N(0,0.02) BF16)",
    }
    config = dict(workload_config(args))
    config["l2"] = "flushed (256 MiB write) before every step"
    if shard:
        gathered_step_ms = g_total / args.steps
        moved = (world - 1) * M * N * 2  # bytes each rank receives
        link_floor_ms = moved / 770e9 * 1e3  # measured peer copy, 770 GB/s per direction
        line.update({
            "value": round(job_flops / (gathered_step_ms * 1e-3) / 1e12, 2),
            "ms_per_step": round(gathered_step_ms, 4),
            "scaling": "strong",
        })
        config.update({"rows_per_gpu": M, "chunks": args.chunks,
                       "parallelism": f"rows sharded x{world}, packed weight replicated, output gathered "
                                      + {"p2p": "by the reconstruct storing into NVLink peer memory",
                                         "ce": "by copy-engine copies into NVLink peer memory, overlapped "
                                               "with the next chunk",
                                         "nccl": "by NCCL all-gather overlapped with the next chunk"}[args.transport]})
        line["no_gather"] = {
            "value": round(job_flops / (local_step_ms * 1e-3) / 1e12, 2),
            "ms_per_step": round(local_step_ms, 4),
            "what": "every rank keeps its own rows of C (no data-path collective)",
        }
        line["gathered"] = {
            "transport": args.transport, "chunks": args.chunks, "reserve_sms": args.reserve_sms,
            "ms_per_step": round(gathered_step_ms, 4),
            "bytes_received_per_gpu": moved,
            "received_gbs": round(moved / (gathered_step_ms * 1e-3) / 1e9, 1),
            "link_floor_ms": round(link_floor_ms, 4),
            "gather_overhead_ms": round(gathered_step_ms - local_step_ms, 4),
            "limiter": (f"every GPU receives (N-1)/N of C: {moved / 1e9:.2f} GB, link floor "
                        f"{link_floor_ms:.3f} ms at the 770 GB/s measured peer copy; the gather adds "
                        f"{gathered_step_ms - local_step_ms:.3f} ms to the {local_step_ms:.3f} ms no-gather step; "
                        + ("the link floor exceeds the no-gather step, so NVLink receive bandwidth bounds it"
                           if link_floor_ms > local_step_ms else
                           "compute exceeds the link floor, so the overhead is the part of the transfer "
                           "not hidden behind the gathering reconstruct")),
        }
        clock_summary = gathered_line["clock"]
    else:
        line.update({
            "value": round(job_flops / (local_step_ms * 1e-3) / 1e12, 2),
            "ms_per_step": round(local_step_ms, 4),
            "scaling": "weak",
        })
        config["parallelism"] = f"replicas x{world}" if world > 1 else "single GPU"
        clock_summary = clock
    line["config"] = config
    line["roofline"] = roofline
    line["kernels"] = kernels
    line["cublas_bf16"] = {"ms": round(cub_ms, 4), "tflops": round(flops_rank / (cub_ms * 1e-3) / 1e12, 1),
                           "speedup": round(cub_ms / local_step_ms, 3),
                           "on": "this GPU's rows" if shard else "the whole workload"}
    line["accuracy"] = accuracy
    line["e2e"] = {"value": round(job_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                   "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                   "api": e2e_api, "streams": lanes,
                   "pinned_buffers": "GPU-local NUMA node" if prev_affinity is not None else "default placement"}
    line["clocks"] = clock_summary
    line["gpu_launches"] = launches
    return line


def _emit(line: dict) -> None:
    os.write(_JSON_FD, (json.dumps(line) + "\n").encode())


_JSON_FD = 1


def default_transport(world: int) -> str:
    """Gather transport measured fastest at this GPU count (c5b): at 2 GPUs the
    copy engines (ce 3.21 ms, p2p 3.40), from 3 up the fused reconstruct (at 8:
    p2p 2.75 ms, ce 3.83-4.85 -- the copy engines do not keep up with seven
    peers at once)."""
    return "ce" if world == 2 else "p2p"


def default_chunking(transport: str, world: int) -> tuple[int, int]:
    """(row chunks per rank, SMs the GEMM leaves free) per gather transport.
    NCCL and the copy engines overlap chunk c's gather with chunk c + 1 (NCCL
    measured best with 32 SMs left to it).  The fused reconstruct from 3 GPUs
    up runs 4 chunks with 48 SMs reserved: its bulk-copy gather kernel takes
    exactly the reserved SMs beside the next chunk's GEMM.  In the per-GPU load
    of the 4- and 8-GPU c5b step, emulated on 2 GPUs, that took 2.825 -> 2.405 ms
    and 2.575 -> 2.312 ms against one chunk with the register gather kernel
    (24-32 reserved SMs, or 2 chunks, gained less or lost).  At 2 GPUs the
    step is compute-bound and p2p keeps one chunk."""
    if transport == "p2p":
        return (4, 48) if world >= 3 else (1, 0)
    return 4, 32


def workload_config(args) -> dict:
    """The workload keys both arms report (the same dict for the same flags)."""
    scheme, M, K, N, with_bias, prepacked, description = WORKLOADS[args.workload]
    if args.rows:
        M = args.rows
        description += f" (rows overridden to {M})"
    return {"workload": f"{args.workload}: {description}", "scheme": scheme, "M": M, "K": K, "N": N,
            "bias": with_bias, "prepacked": prepacked}


def reference_arm(args) -> None:
    """The reference's algorithm on the host cores (CPU oracle, all threads):
    each step one bounded sample; at most 5 so the arm ends within minutes."""
    samples = [cpu_sample(args.workload, target_seconds=4.0) for _ in range(min(args.steps, 5))]
    value = statistics.median(s["value"] for s in samples)
    base = dict(samples[0])
    base["value"] = value
    _emit({
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 and not args.replicas else "weak", "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 leaves", "data": "synthetic",
        "config": {**workload_config(args),
                   "parallelism": "the reference's algorithm on the host cores (rank 0 alone)"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })


def main() -> None:
    global _JSON_FD
    # libraries (NCCL's version banner, for one) may write to stdout; keep
    # the real stdout for the single JSON line and send everything else to stderr
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    parser.add_argument("--impl", default="native", choices=["native", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--rows", type=int, default=0,
                        help="override M (smaller cases for profiler captures)")
    parser.add_argument("--replicas", action="store_true",
                        help="with N GPUs, run one full copy of the workload per GPU (weak scaling) "
                             "instead of sharding its rows")
    parser.add_argument("--e2e-lanes", type=int, default=2,
                        help="streams the single-GPU e2e steps alternate over, each with its own buffers, "
                             "so one step's host->device copies overlap the previous step's compute "
                             "and device->host copy (1: strictly one step after another)")
    parser.add_argument("--no-numa-bind", action="store_true",
                        help="leave the e2e pinned buffers wherever the default policy puts them")
    parser.add_argument("--chunks", type=int, default=None,
                        help="row chunks per rank when sharded (default: 4, which overlaps each "
                             "chunk's gather with the next chunk; 1 with --transport p2p on 2 GPUs)")
    parser.add_argument("--reserve-sms", type=int, default=None,
                        help="SMs the GEMM leaves free, while sharded chunks compute, for the NCCL "
                             "all-gather or the gathering reconstruct of the previous chunk "
                             "(default: 48 for p2p, 32 for NCCL)")
    parser.add_argument("--transport", choices=("nccl", "p2p", "ce"), default=None,
                        help="sharded gather: NCCL all-gather, the reconstruct kernel storing "
                             "into every rank's peer-mapped buffer over NVLink (p2p), or copy-engine "
                             "copies into the peers' buffers behind each chunk (ce); default: the "
                             "fastest measured at that GPU count (ce at 2 GPUs, p2p from 3 up)")
    parser.add_argument("--profile", action="store_true",
                        help="timed steps only: no cuBLAS, e2e or CPU legs")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.transport is None:
        args.transport = default_transport(int(os.environ.get("WORLD_SIZE", "1")))
    default_chunks, default_reserve = default_chunking(args.transport, int(os.environ.get("WORLD_SIZE", "1")))
    if args.chunks is None:
        args.chunks = default_chunks
    if args.reserve_sms is None:
        args.reserve_sms = default_reserve

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            reference_arm(args)
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
            if not args.no_cpu_baseline and world == 1:
                cpu = cpu_sample(args.workload)
                line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
            _emit(line)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
