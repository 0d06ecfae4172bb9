"""Host-side pieces of ``bench.py``: the reference arm's JSON line carries the
contract's keys and reports the same workload configuration as the native arm,
and the sharded run's default gather transport follows the measurements."""

import argparse
import importlib.util
import json
import os
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _args(**overrides):
    base = dict(workload="c5b", rows=0, steps=2, warmup=3, gpus=1, replicas=False)
    base.update(overrides)
    return argparse.Namespace(**base)


def test_default_transport_follows_the_measurements():
    bench = _bench()
    assert bench.default_transport(2) == "ce"
    assert bench.default_transport(4) == "p2p"
    assert bench.default_transport(8) == "p2p"


def test_default_chunking_follows_the_measurements():
    bench = _bench()
    assert bench.default_chunking("p2p", 8) == (4, 48)
    assert bench.default_chunking("p2p", 4) == (4, 48)
    assert bench.default_chunking("p2p", 2) == (1, 0)
    assert bench.default_chunking("nccl", 8) == (4, 32)
    assert bench.default_chunking("ce", 2) == (4, 32)


def test_workload_config_is_the_benchmark_configuration():
    bench = _bench()
    config = bench.workload_config(_args())
    assert config == {"workload": "c5b: " + bench.WORKLOADS["c5b"][6], "scheme": "rank48",
                      "M": 65536, "K": 4608, "N": 12288, "bias": False, "prepacked": True}
    assert bench.workload_config(_args(rows=8192))["M"] == 8192


def test_reference_arm_line(monkeypatch):
    bench = _bench()
    fake = {"value": 0.25, "unit": "TFLOP/s", "cores": 8, "kind": "port", "sample": "fake sample",
            "seconds": 1.0, "rows": 64}
    monkeypatch.setattr(bench, "cpu_sample", lambda workload, target_seconds=4.0: dict(fake))
    read, write = os.pipe()
    monkeypatch.setattr(bench, "_JSON_FD", write)
    bench.reference_arm(_args(gpus=2))
    os.close(write)
    with os.fdopen(read) as stream:
        line = json.loads(stream.read().strip())
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["value"] == 0.25 and line["unit"] == "TFLOP/s" and line["n_gpus"] == 2
    assert line["scaling"] == "strong"
    assert {k: line["config"][k] for k in bench.workload_config(_args())} == bench.workload_config(_args())
    assert line["cpu_baseline"] == {k: fake[k] for k in ("value", "unit", "cores", "kind", "sample")}
    assert line["e2e"] == {"value": 0.25, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
