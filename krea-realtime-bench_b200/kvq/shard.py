"""Head-parallel sharding of the int4-KV attention across GPUs.

The 40 heads are split in contiguous ranges over the ranks (40/20/10/5 per GPU
on 1/2/4/8 B200s); each rank holds the cache of its heads only and runs the
attention for them on all streams. The outputs are all-gathered either by the
attention kernel itself (PeerOutputs: every rank's full-width output buffer is
mapped into every other rank, and the epilogue stores each output row into all
of them over NVLink) or by one NCCL all-gather (gather_outputs). The reference
is single-GPU throughout, so this module has no counterpart there.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_range(n_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced head range [h0, h1) of `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n_heads < world:
        raise ValueError(f"{n_heads} heads cannot be split over {world} ranks")
    base, extra = divmod(n_heads, world)
    h0 = rank * base + min(rank, extra)
    return h0, h0 + base + (1 if rank < extra else 0)


def gather_buffer(local_out: torch.Tensor, world: int) -> torch.Tensor:
    """Receive buffer for gather_outputs(): [world * B, Lq, Hl, D], i.e. the
    per-rank outputs concatenated along the first dimension."""
    return torch.empty((world * local_out.shape[0], *local_out.shape[1:]), dtype=local_out.dtype,
                       device=local_out.device)


def gather_outputs(local_out: torch.Tensor, buf: torch.Tensor | None = None, group=None) -> torch.Tensor:
    """All-gathers per-rank outputs [B, Lq, Hl, D] into [world, B, Lq, Hl, D].

    Equal head counts per rank are required (all_gather_into_tensor). The
    result is rank-major: rank r's heads are head_range(H, world, r).
    """
    world = dist.get_world_size(group)
    if buf is None:
        buf = gather_buffer(local_out, world)
    dist.all_gather_into_tensor(buf, local_out.contiguous(), group=group)
    return buf.view(world, *local_out.shape)


def assemble_heads(gathered: torch.Tensor) -> torch.Tensor:
    """[world, B, Lq, Hl, D] -> [B, Lq, world*Hl, D] in global head order."""
    w, B, Lq, Hl, D = gathered.shape
    return gathered.permute(1, 2, 0, 3, 4).reshape(B, Lq, w * Hl, D)


class PeerOutputs:
    """A full-width output buffer [B, Lq, H, D] bf16 on every rank, mapped into
    every other rank (CUDA IPC), for ops.attention_packed_gather(). `ptrs` lists
    the buffers rank by rank, this rank's own first-hand pointer included.

    Completion without a host barrier: `signal` is a 32-bit counter in this
    rank's memory and `sig_ptrs` lists every rank's counter (mapped like the
    buffers). After each rank's gather launch of a step, `barrier()` on the same
    stream (ops.gather_barrier) adds 1 to every rank's counter once the launch has
    completed and waits on the device until all ranks have done so; work after it
    on the stream reads the whole step's output from `local`. Without signals,
    order the step on the host instead: a stream synchronize on every rank, then
    a barrier.

    Reuse: a rank may store into the buffers again only once every rank has
    finished reading the previous step's `local`. Alternate two PeerOutputs (a
    rank that passed barrier() of step s knows that every rank finished the work
    it ordered before its own step-s barrier, e.g. its reads of step s-1), or put
    a barrier before the next launch.

    `exchange` is the collective that gathers one picklable object per rank
    (dist.all_gather_object by default); `ops` provides ipc_export / ipc_import /
    ipc_close (both replaceable for tests without GPUs)."""

    def __init__(self, local: torch.Tensor, group=None, exchange=None, ops=None, signals: bool = True):
        if ops is None:
            from . import ops as _ops
            ops = _ops
        self._ops = ops
        self.local = local
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if exchange is None:
            def exchange(obj):
                got = [None] * world
                dist.all_gather_object(got, obj, group=group)
                return got
        # the counter gets an allocation of its own (a page), so that its IPC
        # mapping never aliases the output buffer's
        self.signal = torch.zeros(64, dtype=torch.int32, device=local.device) if signals else None
        self.target = 0
        self.world, self.rank = world, rank
        mine = (ops.ipc_export(local), ops.ipc_export(self.signal) if signals else None)
        got = exchange(mine)
        if len(got) != world:
            raise RuntimeError(f"exchange returned {len(got)} entries for {world} ranks")
        self.ptrs: list[int] = []
        self.sig_ptrs: list[int] | None = [] if signals else None
        self._bases: list[int] = []
        try:
            for r, (buf, sig) in enumerate(got):
                if r == rank:
                    self.ptrs.append(local.data_ptr())
                    if signals:
                        self.sig_ptrs.append(self.signal.data_ptr())
                    continue
                base, ptr = ops.ipc_import(*buf)
                self._bases.append(base)
                self.ptrs.append(ptr)
                if signals:
                    base, ptr = ops.ipc_import(*sig)
                    self._bases.append(base)
                    self.sig_ptrs.append(ptr)
        except Exception:
            self.close()
            raise

    def next_target(self) -> int:
        """Advances this rank's barrier target by one barrier (one add per rank)."""
        self.target = (self.target + self.world) & 0xFFFFFFFF
        return self.target

    def barrier(self, wait_cycles: int = 2_000_000_000) -> None:
        """Device-side barrier on the current stream (see the class docstring)."""
        if self.signal is None:
            raise RuntimeError("PeerOutputs made without signals")
        self._ops.gather_barrier(self.sig_ptrs, self.rank, self.next_target(), wait_cycles)

    def close(self) -> None:
        """Unmaps the peers' buffers (call before the peers free theirs)."""
        bases, self._bases = self._bases, []
        for b in bases:
            self._ops.ipc_close(b)
