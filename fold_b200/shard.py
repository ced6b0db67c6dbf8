"""Sequence-sharded far memory over several GPUs (one process per GPU).

The side cache of a layer is partitioned into contiguous position chunks, one per rank
(ShardPlan). Each rank appends only the entries it owns and reads only its chunk with the same
far-read kernel, then folds its split partials into one (o, lse) partial with the combine kernel.
Two ways to combine the per-rank partials:

* "p2p" (the default on GPUs): PeerExchange, one kernel per step that combines this rank's
  splits, stores the result into every rank's receive buffer over NVLink (CUDA IPC mappings of
  one device region per rank), raises a flag per item, waits for the peers' flags and merges
  with the window read. No collective library call on the step.
* "nccl": the combine kernel and one ncclAllGather of the per-rank partials over NVLink, issued by
  the library on the process group's own NCCL communicator (fold_allgather_partials), then the
  merge kernel, which combines any number of partials. Under another torch.distributed backend
  (gloo in the CPU tests) the all-gather is torch's.

The reference runs on one GPU; this module has no counterpart there. The exchange is the only
cross-rank step of the path: the append and the reads are rank-local.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _lib, kernels
from .attention import FoldWorkspace
from .errors import FoldError

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

    @classmethod
    def for_far(cls, length: int, window: int, block: int, world: int, rank: int) -> "ShardPlan":
        """Chunks that split the far keys [0, length - window - block) evenly (whole pages); the last
        rank also holds the positions of the recent window and the block, which the far read does
        not touch."""
        far = max(int(length) - int(window) - int(block), 1)
        chunk = max(SIDE_BLOCK, math.ceil(math.ceil(far / world) / SIDE_BLOCK) * SIDE_BLOCK)
        return cls.even(length, world, rank, chunk)

    @property
    def pos_lo(self) -> int:
        return self.rank * self.chunk  # a rank past the end holds nothing (held == 0)

    @property
    def held(self) -> int:
        if self.rank == self.world - 1:  # the last rank holds everything from its chunk start on
            return max(0, self.length - self.pos_lo)
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


HANDLE_BYTES = 64  # FOLD_EXCHANGE_HANDLE_BYTES


def gather_handles(handle: bytes, group=None, device: Optional[torch.device] = None) -> bytes:
    """All ranks' exchange handles, concatenated in rank order (one all-gather of the bytes; CUDA
    tensors under NCCL, CPU tensors under gloo)."""
    if len(handle) != HANDLE_BYTES:
        raise FoldError(f"an exchange handle has {HANDLE_BYTES} bytes")
    world = dist.get_world_size(group)
    on_cuda = dist.get_backend(group) == "nccl"
    dev = (device or torch.device("cuda", torch.cuda.current_device())) if on_cuda else torch.device("cpu")
    mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
    parts: List[torch.Tensor] = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    return b"".join(bytes(t.cpu().tolist()) for t in parts)


def _slices(hd: int) -> int:
    return hd // 128 if hd > 128 else 1


class PeerExchange:
    """The peer-to-peer exchange of one group of ranks (fold_exchange_* in the C-ABI).

    Created collectively for steps of up to `n` rows, `hq` query heads and head size `hd`; one
    device region per rank (2 parities x world partials + flags) is mapped into every other
    rank. merge() is the step: it replaces combine + all-gather + merge. Every rank must call
    merge() the same number of times with the same shapes, on one stream order."""

    def __init__(self, group=None, *, n: int, hq: int, hd: int, device: Optional[torch.device] = None):
        self.group = group
        # without a process group the exchange is a single rank (its push and wait stay local)
        grouped = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if grouped else 1
        self.rank = dist.get_rank(group) if grouped else 0
        self.n, self.hq, self.hd = int(n), int(hq), int(hd)
        part = self.n * self.hq * self.hd + self.hq * self.n
        part = (part + 3) // 4 * 4
        items = self.n * self.hq * _slices(self.hd)
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        _lib.call("fold_exchange_create", self.world, self.rank, part, items, ctypes.byref(ptr),
                  ctypes.cast(handle, ctypes.c_void_p))
        self._ptr = ptr.value
        try:
            handles = gather_handles(handle.raw, group, device) if grouped else handle.raw
            buf = ctypes.create_string_buffer(handles, len(handles))
            _lib.call("fold_exchange_open", self._ptr, ctypes.cast(buf, ctypes.c_void_p))
            if grouped:
                dist.barrier(group)  # every rank has mapped every region before the first step
        except Exception:
            lib.fold_exchange_destroy(self._ptr)
            self._ptr = None
            raise

    def merge(self, o_part, lse_part, out_l, lse_l, out, qsl, seq_lens, *, window, block, alpha, err=None):
        """Combines this rank's split partials o_part [S, n, Hq, D] / lse_part [S, Hq, n] with every
        other rank's and merges them with the window read into out [n, Hq, D] (bf16)."""
        if self._ptr is None:
            raise FoldError("the exchange is closed")
        kernels._require_cuda(o_part, lse_part, out_l, lse_l, out, qsl, seq_lens, err)
        kernels._check_lengths(qsl, seq_lens)
        s, n, hq, d = o_part.shape
        if (n, hq, d) != tuple(out_l.shape) or tuple(out.shape) != (n, hq, d):
            raise FoldError("exchange merge: o_part, out_l and out shapes differ")
        if n > self.n or hq != self.hq or d != self.hd:
            raise FoldError("exchange merge: the step is larger than the exchange was created for")
        if not o_part.is_contiguous() or not lse_part.is_contiguous() or o_part.dtype != torch.float32 \
                or lse_part.dtype != torch.float32 or tuple(lse_part.shape) != (s, hq, n):
            raise FoldError("exchange merge: partials must be contiguous float32 [S, n, Hq, D] and [S, Hq, n]")
        if out_l.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or lse_l.dtype != torch.float32:
            raise FoldError("exchange merge: out_l and out must be bfloat16 and lse_l float32")
        if out_l.stride(-1) != 1 or out.stride(-1) != 1:
            raise FoldError("exchange merge: the head dimension must be contiguous")
        p = kernels._p
        _lib.call("fold_exchange_merge", self._ptr, p(o_part), p(lse_part), s, p(out_l), out_l.stride(0),
                  out_l.stride(1), p(lse_l), lse_l.stride(0), lse_l.stride(1), p(out), out.stride(0), out.stride(1),
                  p(qsl), p(seq_lens), n, hq, d, int(window), int(block), 1.0 / float(alpha), p(err),
                  kernels._stream(out))
        return out

    def read_merge(self, ws, q, qsl, seq_lens, scale, out_l, lse_l, out, *, rotate=True, err=None):
        """The far read of this rank's chunk (ws.read_far) and merge() in one cooperative launch
        (kernels.far_read_exchange): every CTA of the far read, once all splits of its KV head have
        finished, combines, exchanges and merges a share of that head's items. With one rank it
        is the far read and the merge in one launch. Writes out [n, Hq, D] (bf16)."""
        if self._ptr is None:
            raise FoldError("the exchange is closed")
        n, hq, d = q.shape
        if n > self.n or hq != self.hq or d != self.hd:
            raise FoldError("far read + exchange: the step is larger than the exchange was created for")
        o_part, lse_part = ws.partials(n, hq)
        kernels.far_read_exchange(self._ptr, q, qsl, seq_lens, ws.side, o_part, lse_part, out_l, lse_l, out,
                                  window=ws.window, block=ws.block, far_distance=ws.far_distance,
                                  softmax_scale=scale, alpha=ws.alpha, table=ws.table if rotate else None,
                                  far_len=ws.far_len, pos_lo=ws.pos_lo, capacity=ws.capacity,
                                  err=ws.err if err is None else err)
        return out

    @property
    def handle(self) -> int:
        """The C-ABI handle of the exchange (for kernels.far_read_exchange)."""
        if self._ptr is None:
            raise FoldError("the exchange is closed")
        return self._ptr

    def close(self):
        """Waits for this rank's work, meets the other ranks, then unmaps and frees the region."""
        if self._ptr is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(self.group)
        ptr, self._ptr = self._ptr, None
        _lib.call("fold_exchange_destroy", ptr)


class ShardedFarMemory:
    """The far memory of one layer on one rank of a sharded group.

    step() runs the rank-local far read of this rank's chunk; merge() combines the ranks' partials
    and merges them with the window read (every rank holds the window read and writes the same
    output). exchange="p2p" does the exchange with one PeerExchange kernel (the exchange object
    may be shared by all layers of a group); exchange="nccl" combines the splits in step(),
    all-gathers the per-rank partials there, and merge() applies the merge kernel to them."""

    def __init__(self, plan: ShardPlan, workspace: FoldWorkspace, group=None, *, exchange: str = "p2p",
                 peer: Optional[PeerExchange] = None):
        if exchange not in ("p2p", "nccl"):
            raise FoldError('exchange must be "p2p" or "nccl"')
        self.plan, self.ws, self.group, self.exchange = plan, workspace, group, exchange
        self.peer = peer
        self._bufs = {}
        self._comm_ptr = None

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

    def nccl_comm(self, device) -> int:
        """Address of the group's NCCL communicator on `device` (0 under another backend). The
        first call is collective: a barrier makes sure the communicator exists."""
        if self._comm_ptr is None:
            ptr = 0
            if dist.get_backend(self.group) == "nccl":
                dist.barrier(group=self.group, device_ids=[device.index])
                group = self.group if self.group is not None else dist.group.WORLD
                ptr = int(group._get_backend(device)._comm_ptr())
            self._comm_ptr = ptr
        return self._comm_ptr

    def step(self, q, qsl, seq_lens, scale):
        """p2p: this rank's split partials (o [S, n, Hq, D], lse [S, Hq, n]); nccl: every rank's
        combined partial (o [P, n, Hq, D], lse [P, Hq, n])."""
        n, hq, d = q.shape
        o_part, lse_part = self.ws.read_far(q, qsl, seq_lens, scale)
        if self.exchange == "p2p":
            if self.peer is None:
                self.peer = PeerExchange(self.group, n=n, hq=hq, hd=d, device=q.device)
            return o_part, lse_part
        send, recv, o, lse = self._buffers(n, hq, d, q.device)
        comm = self.nccl_comm(q.device)
        if comm:  # combine + ncclAllGather, issued by the library
            return kernels.allgather_partials(comm, o_part, lse_part, send, recv)
        kernels.combine(o_part, lse_part, o, lse)  # writes straight into the send buffer
        dist.all_gather_into_tensor(recv, send, group=self.group)
        return unpack_partials(recv, self.plan.world, n, hq, d)

    def step_merge(self, q, qsl, seq_lens, scale, out_l, lse_l, out, *, fused=False):
        """step() and merge() of one draft step. fused=True (exchange="p2p" only) runs them as one
        cooperative launch of the far read and the exchange (PeerExchange.read_merge); two launches
        are faster on B200 (the fused kernel's tail costs its far-read loop a few per cent)."""
        if self.exchange == "p2p" and fused:
            n, hq, d = q.shape
            if self.peer is None:
                self.peer = PeerExchange(self.group, n=n, hq=hq, hd=d, device=q.device)
            return self.peer.read_merge(self.ws, q, qsl, seq_lens, scale, out_l, lse_l, out)
        o_all, lse_all = self.step(q, qsl, seq_lens, scale)
        return self.merge(out_l, lse_l, o_all, lse_all, out, qsl, seq_lens)

    def merge(self, out_l, lse_l, o_all, lse_all, out, qsl, seq_lens):
        if self.exchange == "p2p":
            return self.peer.merge(o_all, lse_all, out_l, lse_l, out, qsl, seq_lens, window=self.ws.window,
                                   block=self.ws.block, alpha=self.ws.alpha, err=self.ws.err)
        kernels.merge(out_l, lse_l, o_all, lse_all, out, qsl, seq_lens, window=self.ws.window, block=self.ws.block,
                      alpha=self.ws.alpha)
        return out
