"""Sequence-sharded far memory over several GPUs (one process per GPU).

The side cache of a layer is partitioned into contiguous position chunks, one per rank
(ShardPlan). Each rank appends only the entries it owns and reads only its chunk with the same
far-read kernel, then folds its split partials into one (o, lse) partial with the combine kernel.
The per-rank partials are exchanged with one all-gather (NCCL over NVLink on GPUs; any
torch.distributed backend works, gloo in the CPU tests) and merged with the window read by the
same merge kernel, which combines any number of partials.

The reference runs on one GPU; this module has no counterpart there. The exchange is the only
collective of the path: the append and the reads are rank-local.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import kernels
from .attention import FoldWorkspace

SIDE_BLOCK = kernels.SIDE_BLOCK


@dataclass(frozen=True)
class ShardPlan:
    """Rank `rank` of `world` holds positions [pos_lo, pos_lo + held) of a cache of `length`
    positions; chunks are whole side-cache pages."""

    length: int
    world: int
    rank: int
    chunk: int

    @classmethod
    def even(cls, length: int, world: int, rank: int, chunk: Optional[int] = None) -> "ShardPlan":
        if world < 1 or not 0 <= rank < world:
            raise ValueError("bad world size or rank")
        if chunk is None:
            chunk = math.ceil(math.ceil(length / world) / SIDE_BLOCK) * SIDE_BLOCK
        if chunk % SIDE_BLOCK or chunk < SIDE_BLOCK:
            raise ValueError("shard chunks must be whole 256-entry pages")
        return cls(int(length), int(world), int(rank), int(chunk))

    @property
    def pos_lo(self) -> int:
        return self.rank * self.chunk  # a rank past the end holds nothing (held == 0)

    @property
    def held(self) -> int:
        return max(0, min(self.chunk, self.length - self.pos_lo))

    def owner(self, pos: int) -> int:
        return min(int(pos) // self.chunk, self.world - 1)

    def workspace(self, cache, window, block, *, inv_freq, far_distance, alpha=2.0, num_heads=None, splits=None):
        """The FoldWorkspace of this rank's chunk."""
        return FoldWorkspace(cache, window, block, self.length, inv_freq=inv_freq, far_distance=far_distance,
                             alpha=alpha, num_heads=num_heads, splits=splits, pos_lo=self.pos_lo,
                             shard_len=max(self.held, 1))


def pack_partial(o: torch.Tensor, lse: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One float32 buffer holding o [n, Hq, D] then lse [Hq, n]."""
    flat = torch.cat((o.reshape(-1), lse.reshape(-1))) if out is None else out
    if out is not None:
        out[: o.numel()].copy_(o.reshape(-1))
        out[o.numel():].copy_(lse.reshape(-1))
    return flat


def unpack_partials(buf: torch.Tensor, world: int, n: int, hq: int, d: int):
    """[world * (n*hq*d + hq*n)] -> (o [world, n, Hq, D], lse [world, Hq, n]) views."""
    per = n * hq * d + hq * n
    b = buf.view(world, per)
    return b[:, : n * hq * d].view(world, n, hq, d), b[:, n * hq * d:].view(world, hq, n)


def exchange_partials(o: torch.Tensor, lse: torch.Tensor, group=None, *, send: Optional[torch.Tensor] = None,
                      recv: Optional[torch.Tensor] = None):
    """All-gather every rank's partial. Returns (o_all [P, n, Hq, D], lse_all [P, Hq, n])."""
    world = dist.get_world_size(group)
    n, hq, d = o.shape
    send = pack_partial(o, lse, send)
    if recv is None:
        recv = torch.empty(world * send.numel(), device=send.device, dtype=send.dtype)
    dist.all_gather_into_tensor(recv, send, group=group)
    return unpack_partials(recv, world, n, hq, d)


class ShardedFarMemory:
    """The far memory of one layer on one rank of a sharded group.

    step() runs the rank-local far read of this rank's chunk, combines its splits and all-gathers
    the per-rank partials; merge() applies the merge kernel to the gathered partials and the
    window read (rank 0 holds the window read; any rank may merge)."""

    def __init__(self, plan: ShardPlan, workspace: FoldWorkspace, group=None):
        self.plan, self.ws, self.group = plan, workspace, group
        self._bufs = {}

    def _buffers(self, n, hq, d, device):
        key = (n, hq, d)
        if key not in self._bufs:
            per = n * hq * d + hq * n
            send = torch.empty(per, device=device, dtype=torch.float32)
            recv = torch.empty(self.plan.world * per, device=device, dtype=torch.float32)
            o = send[: n * hq * d].view(n, hq, d)
            lse = send[n * hq * d:].view(hq, n)
            self._bufs[key] = (send, recv, o, lse)
        return self._bufs[key]

    def append(self, k, v, positions, slots):
        self.ws.append(k, v, positions, slots)

    def step(self, q, qsl, seq_lens, scale):
        n, hq, d = q.shape
        send, recv, o, lse = self._buffers(n, hq, d, q.device)
        o_part, lse_part = self.ws.read_far(q, qsl, seq_lens, scale)
        kernels.combine(o_part, lse_part, o, lse)  # writes straight into the send buffer
        dist.all_gather_into_tensor(recv, send, group=self.group)
        return unpack_partials(recv, self.plan.world, n, hq, d)

    def merge(self, out_l, lse_l, o_all, lse_all, out, qsl, seq_lens):
        kernels.merge(out_l, lse_l, o_all, lse_all, out, qsl, seq_lens, window=self.ws.window, block=self.ws.block,
                      alpha=self.ws.alpha)
        return out
