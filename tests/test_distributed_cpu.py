"""Host logic of the row-sharded linear on 2 CPU ranks (gloo): sharding
arithmetic, in-place all-gather assembly, and a failed rank turning into an
error on its peer instead of a hang.  The B200 plan is replaced by
``F.linear`` on the CPU (the product is never exercised here)."""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rdna3_fastmm.distributed import RowShardedLinear, shard_rows


def test_shard_rows_even_and_uneven():
    assert shard_rows(8192, 4) == [(0, 2048), (2048, 2048), (4096, 2048), (6144, 2048)]
    assert shard_rows(10, 4) == [(0, 3), (3, 3), (6, 2), (8, 2)]
    assert sum(c for _, c in shard_rows(65537, 8)) == 65537
    with pytest.raises(ValueError):
        shard_rows(0, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, mode, results, chunks=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        g = torch.Generator().manual_seed(0)
        A = torch.randn((rows, 16), generator=g).to(torch.bfloat16)
        W = torch.randn((24, 16), generator=g).to(torch.bfloat16)

        def local(x, out):
            out.copy_(torch.nn.functional.linear(x, W))

        layer = RowShardedLinear(None, rows, W, local_linear=local, chunks=chunks)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 leaves before the collective")
        try:
            full = layer(layer.local_rows(A))
            mine = layer(layer.local_rows(A), gather=False)
            expected = torch.nn.functional.linear(A, W)
            mine_expected = torch.cat([expected[s:s + n] for s, n in layer.row_blocks()])
            results[rank] = bool(torch.equal(full, expected)) and bool(torch.equal(mine, mine_expected))
        except RuntimeError as error:  # the peer is gone: the collective errors out
            results[rank] = f"error: {type(error).__name__}"
    except RuntimeError:
        results[rank] = "left"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, rows, mode, chunks=1):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, mode, results, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    return dict(results)


@pytest.mark.parametrize("rows", [64, 37])
def test_two_rank_gather_matches_full_linear(rows):
    results = _run(2, rows, "ok")
    assert results == {0: True, 1: True}


def test_chunked_block_cyclic_gather_matches_full_linear():
    """4 chunks per rank, gathered asynchronously chunk by chunk."""
    results = _run(2, 64, "ok", chunks=4)
    assert results == {0: True, 1: True}


def test_failed_rank_becomes_an_error_not_a_hang():
    results = _run(2, 64, "fail")
    assert results[1] == "left"
    assert str(results[0]).startswith("error")


def test_transport_arguments_are_validated():
    store = dist.HashStore()
    dist.init_process_group("gloo", store=store, rank=0, world_size=1)
    try:
        W = torch.zeros((8, 4), dtype=torch.bfloat16)

        def local(x, out):
            out.copy_(torch.nn.functional.linear(x, W))

        with pytest.raises(ValueError, match="transport"):
            RowShardedLinear(None, 16, W, local_linear=local, transport="nvshmem")
        for transport in ("p2p", "ce"):
            with pytest.raises(ValueError, match="transports run the B200 plan"):
                RowShardedLinear(None, 16, W, local_linear=local, transport=transport)
        layer = RowShardedLinear(None, 16, W, local_linear=local, transport="nccl")
        assert layer.transport == "nccl"
    finally:
        dist.destroy_process_group()


def test_p2p_chunks_give_the_gather_the_reserved_sms(monkeypatch):
    """With chunks and reserved SMs, each chunk's transform and GEMM are queued
    under the budget that leaves `reserve_sms` SMs free, and its gathering
    reconstruct under a budget of exactly `reserve_sms` (the kernel runs one
    CTA per SM), so it runs beside the next chunk's GEMM.  The budget is
    released afterwards.  CUDA streams, events and the library are replaced
    by recorders: this pins the host-side order only."""
    import contextlib
    from types import SimpleNamespace

    from rdna3_fastmm import _native

    log, budget = [], [0]
    monkeypatch.setattr(_native, "set_sm_budget", lambda n: budget.__setitem__(0, n))
    monkeypatch.setattr(_native, "transform_a", lambda *a: log.append(("transform", budget[0])))
    monkeypatch.setattr(_native, "leaf_gemm", lambda *a: log.append(("gemm", budget[0])))
    monkeypatch.setattr(_native, "reconstruct_gather", lambda *a: log.append(("gather", budget[0])))

    class Event:
        def record(self, stream=None):
            pass

    class Stream:
        def wait_event(self, event):
            pass

    monkeypatch.setattr(torch.cuda, "Event", Event)
    monkeypatch.setattr(torch.cuda, "stream", lambda stream: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda device: SimpleNamespace(multi_processor_count=148))
    layer = object.__new__(RowShardedLinear)
    layer.plan = SimpleNamespace(scheme="rank48", rank=48,
                                 shape=SimpleNamespace(block_rows=512, block_columns=3072, block_inner=1152))
    layer.workspace = SimpleNamespace(left_transformed=None)
    layer.packed = SimpleNamespace(transformed=None)
    layer._products = [object(), object()]
    layer.world, layer.rank, layer.chunks, layer.chunk_rows = 2, 0, 4, 2048
    layer.reserve_sms, layer.device, layer.columns, layer.bias = 48, "cpu", 12288, None
    layer._side = Stream()
    layer._peer_bases = [0, 1 << 40]
    reserved = layer._reserve()
    layer._p2p_chunks(torch.zeros((4 * 2048, 8)), Stream(), 12288 * 2, [None, None], reserved)
    layer._release(reserved)
    assert log == [("transform", 100), ("gemm", 100), ("gather", 48)] * 4
    assert budget[0] == 0
