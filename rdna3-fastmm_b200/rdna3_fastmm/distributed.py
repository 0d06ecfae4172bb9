"""Row-sharded reduced-rank linear over one process per GPU.

Rows of ``A`` are independent, so a large-M linear splits into per-rank row
blocks with no data exchange: every rank packs the (replicated) weight once,
transforms its own rows and writes its own rows of ``C``.  The only exchange
is optional: when the caller needs the whole ``C[M, N]`` on every rank, the row
blocks are all-gathered over NCCL (NVLink / NVSwitch).  Each rank writes its
rows straight into its slot of the gather buffer and the all-gather runs in
place, so no extra copy is made.

The reference is single-GPU; this is the multi-GPU form north_star asks for
(M sharded across 1/2/4/8 GPUs, weight replicated, all-gather on demand).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

__all__ = ["shard_rows", "RowShardedLinear"]


def shard_rows(rows: int, world: int) -> list[tuple[int, int]]:
    """(start, count) of every rank's row block: even split, the first
    ``rows % world`` ranks take one extra row."""
    if rows < 1 or world < 1:
        raise ValueError("rows and world size must be positive")
    base, extra = divmod(rows, world)
    out, start = [], 0
    for r in range(world):
        count = base + (1 if r < extra else 0)
        out.append((start, count))
        start += count
    return out


@dataclass
class _Shard:
    start: int
    count: int
    padded: int  # rows of every slot in the gather buffer


class RowShardedLinear:
    """``C = A @ weight^T (+ bias)`` with rows of ``A`` split over a process group.

    ``plan_type`` is one of the rank plans; ``weight`` is the full native
    ``[N, K]`` weight, replicated on every rank and packed locally.  ``local_linear``
    replaces the B200 plan for host-logic tests (it receives the local rows and
    must return ``[count, N]``).
    """

    def __init__(self, plan_type, rows: int, weight: torch.Tensor, *, group=None,
                 bias: Optional[torch.Tensor] = None,
                 local_linear: Optional[Callable[[torch.Tensor, torch.Tensor], None]] = None,
                 max_free_memory_fraction: float = 0.75) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.columns, self.inner = weight.shape
        self.rows = rows
        start, count = shard_rows(rows, self.world)[self.rank]
        self.shard = _Shard(start, count, -(-rows // self.world))
        self.bias = bias
        self.device = weight.device
        if local_linear is not None:
            self._local = local_linear
            self.plan = None
        else:
            self.plan = plan_type(count, self.inner, self.columns, weight.device,
                                  dtype=weight.dtype, compute_dtype=torch.float16)
            self.packed = self.plan.pack_weight(weight, max_free_memory_fraction)
            self.workspace = self.plan.allocate_workspace(max_free_memory_fraction, prepacked_right=True)
            self._local = self._plan_linear

    def _plan_linear(self, local_rows: torch.Tensor, out: torch.Tensor) -> None:
        self.plan.run_linear_packed(local_rows, self.packed, self.workspace, self.bias, out)

    def local_rows(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's rows of a full ``[M, K]`` input (a view)."""
        return full[self.shard.start:self.shard.start + self.shard.count]

    def gather_buffer(self) -> torch.Tensor:
        return torch.empty((self.world * self.shard.padded, self.columns), device=self.device,
                           dtype=torch.bfloat16)

    def __call__(self, local_rows: torch.Tensor, *, gather: bool = True,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Run this rank's rows; with ``gather`` return the whole ``C[M, N]``
        on every rank, else this rank's ``[count, N]`` rows."""
        if tuple(local_rows.shape) != (self.shard.count, self.inner):
            raise ValueError(f"local rows have shape {tuple(local_rows.shape)}, "
                             f"expected {(self.shard.count, self.inner)}")
        if not gather:
            result = out if out is not None else torch.empty(
                (self.shard.count, self.columns), device=self.device, dtype=torch.bfloat16)
            self._local(local_rows, result)
            return result
        full = out if out is not None else self.gather_buffer()
        if tuple(full.shape) != (self.world * self.shard.padded, self.columns):
            raise ValueError("gather buffer does not match the sharding")
        slot = full[self.rank * self.shard.padded:(self.rank + 1) * self.shard.padded]
        self._local(local_rows, slot[: self.shard.count])
        if self.shard.count < self.shard.padded:
            slot[self.shard.count:].zero_()
        dist.all_gather_into_tensor(full, slot, group=self.group)
        if self.rows == self.world * self.shard.padded:
            return full
        # uneven split: drop the padding rows of the short slots
        pieces = [full[r * self.shard.padded:r * self.shard.padded + c]
                  for r, (_, c) in enumerate(shard_rows(self.rows, self.world))]
        return torch.cat(pieces)
