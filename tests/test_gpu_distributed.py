"""Row-sharded linear on 2 B200s (skipped with fewer GPUs): the fused
reconstruct + all-gather over NVLink peer memory (``transport="p2p"``, CUDA
IPC mappings) and the copy-engine gather (``transport="ce"``) must give bit for
bit the rows of the reconstruct + NCCL all-gather path, on every rank, with and
without chunking and bias."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, case: tuple, results) -> None:
    """Every rank runs to the end and tears down collectively (no rank leaves
    while a peer may still write into its buffer); the parent asserts."""
    from inputs import make_linear_inputs
    from rdna3_fastmm.distributed import RowShardedLinear
    from rdna3_fastmm.runtime import Rank7Plan, Rank48Plan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=device)
    p2p = ce = None
    try:
        scheme, M, K, N, chunks, with_bias, *more = case
        reserve = more[0] if more else 0
        plan_type = {"rank7": Rank7Plan, "rank48": Rank48Plan}[scheme]
        A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=with_bias)
        A, W = A.to(device), W.to(device)
        bias = bias.to(device) if bias is not None else None
        nccl = RowShardedLinear(plan_type, M, W, bias=bias, chunks=chunks)
        p2p = RowShardedLinear(plan_type, M, W, bias=bias, chunks=chunks, transport="p2p", reserve_sms=reserve)
        ce = RowShardedLinear(plan_type, M, W, bias=bias, chunks=chunks, transport="ce")
        rows = nccl.local_rows(A)
        expected = nccl(rows)[:M].clone()
        got = p2p(rows).clone()
        got2 = p2p(rows).clone()  # the second call reuses the mapped buffers
        got_ce = ce(rows).clone()
        got_ce2 = ce(rows).clone()
        torch.cuda.synchronize()
        ref = torch.nn.functional.linear(A.float(), W.float(), None if bias is None else bias.float())
        err = float(torch.linalg.vector_norm(got.float() - ref) / torch.linalg.vector_norm(ref))
        results[rank] = {
            "shape": tuple(got.shape) == (M, N),
            "equal": bool(torch.equal(got.view(torch.int16), expected.view(torch.int16))),
            "equal_again": bool(torch.equal(got2.view(torch.int16), expected.view(torch.int16))),
            "ce_equal": bool(torch.equal(got_ce.view(torch.int16), expected.view(torch.int16))
                             and torch.equal(got_ce2.view(torch.int16), expected.view(torch.int16))),
            "err": err,
        }
    finally:
        for layer in (p2p, ce):
            if layer is not None:
                layer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("case", [
    ("rank48", 1024, 512, 768, 1, False),
    ("rank48", 1024, 512, 768, 2, True),
    ("rank7", 1030, 384, 520, 1, True),
    # chunks with SMs reserved: each chunk's gather runs on the reserved SMs
    # beside the next chunk's GEMM on the others
    ("rank48", 4096, 512, 1536, 4, True, 32),
], ids=lambda c: "-".join(map(str, c)))
def test_p2p_gather_matches_nccl_gather(case):
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(2, _free_port(), case, results), nprocs=2, join=True)
        results = dict(results)
    for rank in range(2):
        r = results[rank]
        assert r["shape"] and r["equal"] and r["equal_again"] and r["ce_equal"], (rank, case, r)
        assert r["err"] < 5e-3, (rank, case, r)
