"""Row-sharded linear on 2 B200s (skipped with fewer GPUs): the fused
reconstruct + all-gather over NVLink peer memory (``transport="p2p"``) must
give bit for bit the rows of the reconstruct + NCCL all-gather path, on every
rank, with and without chunking and bias."""

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


def _worker(rank: int, world: int, port: int, case: tuple) -> None:
    from inputs import make_linear_inputs
    from rdna3_fastmm.distributed import RowShardedLinear
    from rdna3_fastmm.runtime import Rank7Plan, Rank48Plan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=device)
    try:
        scheme, M, K, N, chunks, with_bias = case
        plan_type = {"rank7": Rank7Plan, "rank48": Rank48Plan}[scheme]
        A, W, bias = make_linear_inputs(M, K, N, seed=0, bias=with_bias)
        A, W = A.to(device), W.to(device)
        bias = bias.to(device) if bias is not None else None
        nccl = RowShardedLinear(plan_type, M, W, bias=bias, chunks=chunks)
        p2p = RowShardedLinear(plan_type, M, W, bias=bias, chunks=chunks, transport="p2p")
        rows = nccl.local_rows(A)
        expected = nccl(rows).clone()
        got = p2p(rows).clone()
        torch.cuda.synchronize()
        assert got.shape == (M, N)
        assert torch.equal(got.view(torch.int16), expected[:M].view(torch.int16)), (rank, case)
        # a second call reuses the symmetric buffer
        got2 = p2p(rows)
        torch.cuda.synchronize()
        assert torch.equal(got2.view(torch.int16), expected[:M].view(torch.int16))
        ref = torch.nn.functional.linear(A.float(), W.float(), None if bias is None else bias.float())
        err = torch.linalg.vector_norm(got.float() - ref) / torch.linalg.vector_norm(ref)
        assert err < 5e-3
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("case", [
    ("rank48", 1024, 512, 768, 1, False),
    ("rank48", 1024, 512, 768, 2, True),
    ("rank7", 1030, 384, 520, 1, True),
], ids=lambda c: "-".join(map(str, c)))
def test_p2p_gather_matches_nccl_gather(case):
    mp.spawn(_worker, args=(2, _free_port(), case), nprocs=2, join=True)
