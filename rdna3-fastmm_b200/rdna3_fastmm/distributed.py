"""Row-sharded reduced-rank linear over one process per GPU.

Rows of ``A`` are independent, so a large-M linear splits into per-rank row
blocks with no data exchange: every rank packs the (replicated) weight once,
transforms its own rows and writes its own rows of ``C``.  The only exchange
is optional: when the caller needs the whole ``C[M, N]`` on every rank, the row
blocks are all-gathered over NCCL (NVLink / NVSwitch).  Each rank writes its
rows straight into its slot of the gather buffer and the all-gather runs in
place, so no extra copy is made.

With ``chunks > 1`` the rows are dealt out block-cyclically: chunk ``c`` of
rank ``r`` is global row block ``c * world + r`` (``M / (world * chunks)`` rows
each), so chunk ``c`` of every rank forms one contiguous slice of ``C``.  Each
chunk is computed on the current stream and its slice is all-gathered
asynchronously while the next chunk computes, overlapping NVLink traffic with
tensor-core work.

``transport="p2p"`` replaces the reconstruct + NCCL all-gather pair by one
kernel (``fmm_reconstruct_gather``): every rank exports its gather buffer by
CUDA IPC and maps its peers' buffers (plain peer mappings, no multicast
object), and each rank's output transform stores every output vector into its
own buffer and, over NVLink, into every peer's buffer at this rank's rows
(for rank 48/49 with 16-byte-aligned rows: row segments staged in shared
memory and written by bulk async copies, one CTA per SM).  With ``chunks > 1``
the gathering reconstruct of chunk c runs on a side stream while chunk c + 1
transforms and multiplies (two product workspaces alternate).  With
``reserve_sms`` as well, the transform and GEMM are queued under an SM budget
that leaves ``reserve_sms`` SMs free, and the gather under a budget of exactly
``reserve_sms``, so NVLink traffic overlaps tensor-core work on disjoint SMs
(from 3 GPUs up, ``chunks=4, reserve_sms=48`` measured best on c5b).  A
one-element all-reduce queued behind the kernels makes every peer's rows
visible before the result is used.

``transport="ce"`` keeps the reconstruct local (each chunk's rows land in this
rank's own IPC-exported output buffer) and hands the transfer to the copy
engines: one device-to-device copy per peer and chunk (``fmm_copy_async``) on
a stream of its own, into the peer's mapped buffer.  The copies of chunk c run
while chunk c + 1 transforms, multiplies and reconstructs, and no SM is spent
on the transfer; the same all-reduce ends the call.

The reference is single-GPU; this is the path's multi-GPU form (M sharded
across 1/2/4/8 GPUs, weight replicated, output gathered on demand).
"""

from __future__ import annotations

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


class RowShardedLinear:
    """``C = A @ weight^T (+ bias)`` with rows of ``A`` split over a process group.

    ``plan_type`` is one of the rank plans; ``weight`` is the full native
    ``[N, K]`` weight, replicated on every rank and packed locally.  ``chunks``
    (> 1 needs ``rows % (world * chunks) == 0``) overlaps the all-gather with
    compute as described in the module docstring.  ``local_linear`` replaces
    the B200 plan for host-logic tests: it receives ``(rows [n, K], out [n, N])``.
    """

    def __init__(self, plan_type, rows: int, weight: torch.Tensor, *, group=None,
                 bias: Optional[torch.Tensor] = None, chunks: int = 1, reserve_sms: int = 0,
                 local_linear: Optional[Callable[[torch.Tensor, torch.Tensor], None]] = None,
                 max_free_memory_fraction: float = 0.75, transport: str = "nccl") -> None:
        if transport not in ("nccl", "p2p", "ce"):
            raise ValueError("transport must be 'nccl', 'p2p' or 'ce'")
        if transport in ("p2p", "ce") and local_linear is not None:
            raise ValueError("the p2p and ce transports run the B200 plan, not a local stand-in")
        self.transport = transport
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.columns, self.inner = weight.shape
        self.rows = rows
        if chunks < 1:
            raise ValueError("chunks must be positive")
        if chunks > 1 and rows % (self.world * chunks):
            raise ValueError("chunked sharding needs rows divisible by world * chunks")
        self.chunks = chunks
        if chunks > 1:
            self.chunk_rows = rows // (self.world * chunks)
            self.count = self.chunk_rows * chunks
            self.padded = self.count
        else:
            start, self.count = shard_rows(rows, self.world)[self.rank]
            self.start = start
            self.chunk_rows = self.count
            self.padded = -(-rows // self.world)
        self.bias = bias
        self.device = weight.device
        # SMs left to NCCL while chunks compute (0: the library fills them all)
        self.reserve_sms = reserve_sms
        if local_linear is not None:
            self._local = local_linear
            self.plan = None
        else:
            self.plan = plan_type(self.chunk_rows, self.inner, self.columns, weight.device,
                                  dtype=weight.dtype, compute_dtype=torch.float16)
            self.packed = self.plan.pack_weight(weight, max_free_memory_fraction)
            self.workspace = self.plan.allocate_workspace(max_free_memory_fraction, prepacked_right=True)
            self._local = self._plan_linear
        if transport in ("p2p", "ce"):
            self._setup_p2p(max_free_memory_fraction)

    def _setup_p2p(self, max_free_memory_fraction: float) -> None:
        from . import _native

        if self.world > 8:
            raise ValueError("the gathering reconstruct stores to at most 8 ranks")
        if self.bias is not None and self.bias.dtype != torch.bfloat16:
            raise ValueError("bias must be BF16")
        # exact [M, N] rows: every rank writes its own rows, no padding slots
        self._gather_out = torch.empty((self.rows, self.columns), dtype=torch.bfloat16, device=self.device)
        mine = _native.ipc_export(self._gather_out.data_ptr())
        exported: list = [None] * self.world
        dist.all_gather_object(exported, mine, group=self.group)
        self._ipc_bases: list[int] = []
        self._peer_bases: list[int] = []
        for peer, (handle, offset) in enumerate(exported):
            if peer == self.rank:
                self._peer_bases.append(self._gather_out.data_ptr())
            else:
                base, ptr = _native.ipc_import(handle, offset)
                self._ipc_bases.append(base)
                self._peer_bases.append(ptr)
        # a second product workspace so chunk c's gathering reconstruct can
        # read its products while chunk c + 1 multiplies
        self._products = [self.workspace.products]
        if self.chunks > 1 and self.transport == "p2p":
            self._products.append(torch.empty_like(self.workspace.products))
        self._side = torch.cuda.Stream(device=self.device)
        # ce: one copy stream per peer, so the copies to different peers run on
        # separate copy engines at once
        self._copy_streams = ([torch.cuda.Stream(device=self.device) for _ in range(self.world - 1)]
                              if self.transport == "ce" else [])
        self._flag = torch.zeros(1, device=self.device, dtype=torch.int32)

    def close(self) -> None:
        """Unmap the peers' buffers (p2p transport).  Collective: no rank frees
        its gather buffer while a peer could still write into it."""
        if self.transport not in ("p2p", "ce") or not self._ipc_bases:
            return
        from . import _native

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for base in self._ipc_bases:
            _native.ipc_close(base)
        self._ipc_bases = []
        dist.barrier(group=self.group)

    def _p2p(self, local_rows: torch.Tensor) -> torch.Tensor:
        main = torch.cuda.current_stream(self.device)
        row_bytes = self.columns * 2
        done: list = [None] * len(self._products)
        # with chunks the GEMM of chunk c + 1 leaves `reserve_sms` SMs to the
        # gathering reconstruct of chunk c, which runs beside it on those SMs
        budget = self._reserve() if self.chunks > 1 else False
        try:
            self._p2p_chunks(local_rows, main, row_bytes, done, budget)
        finally:
            self._release(budget)
        main.wait_stream(self._side)
        # completion: an all-reduce queued behind the gathering kernels ends on
        # a rank only after every rank's kernels (and their fenced peer
        # stores) have finished; NCCL's process-group timeout bounds the wait
        dist.all_reduce(self._flag, group=self.group)
        return self._gather_out

    def _p2p_chunks(self, local_rows: torch.Tensor, main, row_bytes: int, done: list, reserved: bool) -> None:
        from . import _native

        plan, ws = self.plan, self.workspace
        s = plan.shape
        for c, (start, count) in enumerate(self.row_blocks()):
            k = c % len(self._products)
            P = self._products[k]
            if done[k] is not None:
                main.wait_event(done[k])  # the side stream has finished reading P
            _native.transform_a(plan.scheme, local_rows[c * self.chunk_rows:c * self.chunk_rows + count],
                                ws.left_transformed)
            _native.leaf_gemm(plan.rank, ws.left_transformed, self.packed.transformed, s.block_rows,
                              s.block_columns, s.block_inner, P)
            ready = torch.cuda.Event()
            ready.record(main)
            self._side.wait_event(ready)
            with torch.cuda.stream(self._side):
                dests = [base + start * row_bytes for base in self._peer_bases]
                if reserved:
                    # the budget is read when a launch is queued: the gather
                    # takes the reserved SMs (one CTA each), the next chunk's
                    # transform and GEMM the rest
                    _native.set_sm_budget(self.reserve_sms)
                _native.reconstruct_gather(plan.scheme, P, count, self.columns, self.bias, dests,
                                           self.columns, torch.bfloat16)
                if reserved:
                    self._reserve()
            done[k] = torch.cuda.Event()
            done[k].record(self._side)

    def _ce(self, local_rows: torch.Tensor) -> torch.Tensor:
        from . import _native

        main = torch.cuda.current_stream(self.device)
        row_bytes = self.columns * 2
        own = self._gather_out
        peers = [base for peer, base in enumerate(self._peer_bases) if peer != self.rank]
        ch = self.chunk_rows
        for c, (start, count) in enumerate(self.row_blocks()):
            self._plan_linear(local_rows[c * ch:c * ch + count], own[start:start + count])
            ready = torch.cuda.Event()
            ready.record(main)
            src = own.data_ptr() + start * row_bytes
            for stream, base in zip(self._copy_streams, peers):
                stream.wait_event(ready)
                _native.copy_async(base + start * row_bytes, src, count * row_bytes, stream.cuda_stream)
        for stream in self._copy_streams:
            main.wait_stream(stream)
        # completion: as for p2p, an all-reduce queued behind this rank's copies
        dist.all_reduce(self._flag, group=self.group)
        return own

    def _plan_linear(self, local_rows: torch.Tensor, out: torch.Tensor) -> None:
        self.plan.run_linear_packed(local_rows, self.packed, self.workspace, self.bias, out)

    def _reserve(self) -> bool:
        if self.reserve_sms <= 0 or self.plan is None:
            return False
        from . import _native

        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        _native.set_sm_budget(max(2, sms - self.reserve_sms))
        return True

    def _release(self, reserved: bool) -> None:
        if reserved:
            from . import _native

            _native.set_sm_budget(0)

    def row_blocks(self) -> list[tuple[int, int]]:
        """(start, count) of the global rows this rank owns, in local order."""
        if self.chunks == 1:
            return [(self.start, self.count)]
        ch = self.chunk_rows
        return [((c * self.world + self.rank) * ch, ch) for c in range(self.chunks)]

    def local_rows(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's rows of a full ``[M, K]`` input (contiguous)."""
        blocks = [full[s:s + n] for s, n in self.row_blocks()]
        return blocks[0] if len(blocks) == 1 else torch.cat(blocks)

    def gather_buffer(self) -> torch.Tensor:
        return torch.empty((self.world * self.padded, self.columns), device=self.device,
                           dtype=torch.bfloat16)

    def __call__(self, local_rows: torch.Tensor, *, gather: bool = True,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Run this rank's rows; with ``gather`` return the whole ``C[M, N]``
        on every rank, else this rank's ``[count, N]`` rows (local order).
        With the p2p transport the gathered result is the layer's own gather
        buffer, overwritten by the next call."""
        if tuple(local_rows.shape) != (self.count, self.inner):
            raise ValueError(f"local rows have shape {tuple(local_rows.shape)}, "
                             f"expected {(self.count, self.inner)}")
        ch = self.chunk_rows
        if gather and self.transport in ("p2p", "ce"):
            if out is not None:
                raise ValueError("the p2p and ce transports gather into their own peer-mapped buffer")
            return self._p2p(local_rows) if self.transport == "p2p" else self._ce(local_rows)
        if not gather:
            result = out if out is not None else torch.empty(
                (self.count, self.columns), device=self.device, dtype=torch.bfloat16)
            for c in range(self.chunks):
                self._local(local_rows[c * ch:(c + 1) * ch], result[c * ch:(c + 1) * ch])
            return result
        full = out if out is not None else self.gather_buffer()
        if tuple(full.shape) != (self.world * self.padded, self.columns):
            raise ValueError("gather buffer does not match the sharding")
        if self.chunks > 1:
            handles = []
            span = self.world * ch
            budget = self._reserve()
            try:
                for c in range(self.chunks):
                    region = full[c * span:(c + 1) * span]
                    slot = region[self.rank * ch:(self.rank + 1) * ch]
                    self._local(local_rows[c * ch:(c + 1) * ch], slot)
                    handles.append(dist.all_gather_into_tensor(region, slot, group=self.group,
                                                               async_op=True))
            finally:
                self._release(budget)
            for handle in handles:
                handle.wait()
            return full
        slot = full[self.rank * self.padded:(self.rank + 1) * self.padded]
        self._local(local_rows, slot[: self.count])
        if self.count < self.padded:
            slot[self.count:].zero_()
        dist.all_gather_into_tensor(full, slot, group=self.group)
        if self.rows == self.world * self.padded:
            return full
        # uneven split: drop the padding rows of the short slots
        pieces = [full[r * self.padded:r * self.padded + c]
                  for r, (_, c) in enumerate(shard_rows(self.rows, self.world))]
        return torch.cat(pieces)
