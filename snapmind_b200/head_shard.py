"""KV-head-sharded paged decode across GPUs.

Sequence sharding needs no collective (every rank owns whole sequences).  The
alternative for a batch that must stay on every rank is to shard the KV heads:
rank r keeps kv heads [r*H/N, (r+1)*H/N) of every sequence (and serves the
query heads of those groups), runs the paged GQA decode on its slice, and the
per-layer outputs — disjoint head ranges, so no reduction — are all-gathered:
``B x Hq x D`` elements per layer (1 MiB at B = 128, Hq = 32, D = 128, bf16).

``HeadShardedDecode`` gathers with ``torch.distributed.all_gather_into_tensor``
(NCCL over NVLink on GPUs; gloo works for the host-side tests), followed by one
reorder of the gathered ``[N, B, Hq/N, D]`` into ``[B, Hq, D]``.

``PeerHeadShardedDecode`` fuses the exchange into the decode kernel: its
epilogue stores every finished output row into every rank's ``[B, Hq, D]``
buffer at the row's global head (16-byte NVLink stores through CUDA IPC
mappings), so the rows land in place while other CTAs are still attending.
One warp after it publishes the call's epoch into every rank's flag array and
waits (bounded) for all ranks' epochs.  No collective launch, no gathered
copy, no reorder.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib


def head_range(n_heads: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the heads rank ``rank`` owns; heads split evenly."""
    if n_heads % world != 0:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    per = n_heads // world
    return rank * per, (rank + 1) * per


def shard_query(q: torch.Tensor, n_kv_heads: int, world: int, rank: int) -> torch.Tensor:
    """The query heads of this rank's kv heads: q [B, Hq, D] -> [B, Hq/N, D] (a view)."""
    n_q = q.shape[1]
    group = n_q // n_kv_heads
    lo, hi = head_range(n_kv_heads, world, rank)
    return q[:, lo * group: hi * group]


def gather_heads(local_out: torch.Tensor, world: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather the per-rank head slices [B, Hq/N, D] into [B, Hq, D]."""
    b, hl, d = local_out.shape
    gathered = torch.empty((world, b, hl, d), dtype=local_out.dtype, device=local_out.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local_out.contiguous(), group=group)
    else:  # gloo (host-side tests) has only the list form
        dist.all_gather(list(gathered.unbind(0)), local_out.contiguous(), group=group)
    if out is None:
        out = torch.empty((b, world * hl, d), dtype=local_out.dtype, device=local_out.device)
    out.view(b, world, hl, d).copy_(gathered.permute(1, 0, 2, 3))
    return out


class HeadShardedDecode:
    """Paged GQA decode over a PagedKVPool that holds this rank's kv-head slice."""

    def __init__(self, pool, n_q_heads: int, world: int, rank: int, group=None):
        self.pool, self.world, self.rank, self.group = pool, world, rank, group
        self.n_q_heads = n_q_heads
        self.n_kv_total = pool.n_kv_heads * world
        if n_q_heads % self.n_kv_total != 0:
            raise ValueError("query heads must be a multiple of the kv heads")

    def decode(self, layer: int, q: torch.Tensor, out: torch.Tensor | None = None, **kw) -> torch.Tensor:
        """q [B, Hq, D] (all heads) -> out [B, Hq, D] (all heads, on every rank)."""
        q_local = shard_query(q, self.n_kv_total, self.world, self.rank)
        local = self.pool.decode(layer, q_local, **kw)
        return gather_heads(local, self.world, self.group, out)


@dataclass
class PeerTargets:
    """Destinations of one head-sharded decode call (``PagedKVPool.decode(peers=...)``)."""

    out_ptrs: torch.Tensor   # int64 [n] device: each rank's output base for this call
    n: int
    head_offset: int         # global index of this rank's first query head
    out_stride_seq: int      # elements
    out_stride_head: int


# allocations opened in this process: handle bytes -> [base pointer, users]
_OPENED: dict[bytes, list] = {}


def _ipc_open(handle: bytes, offset: int) -> int:
    ent = _OPENED.get(handle)
    if ent is None:
        ptr = ctypes.c_void_p()
        _lib.check(_lib.load().snapmind_ipc_open(handle, 0, ctypes.byref(ptr)), "snapmind_ipc_open")
        ent = _OPENED[handle] = [ptr.value, 0]
    ent[1] += 1
    return ent[0] + offset


def _ipc_release(handle: bytes) -> None:
    ent = _OPENED[handle]
    ent[1] -= 1
    if ent[1] == 0:
        del _OPENED[handle]
        _lib.check(_lib.load().snapmind_ipc_close(ent[0], 0), "snapmind_ipc_close")


class PeerHeadShardedDecode(HeadShardedDecode):
    """Head-sharded decode whose kernel writes the outputs of every rank directly.

    Each rank owns one device buffer holding two ``[max_batch, Hq, D]`` receive
    buffers and an int32 flag per rank; the ranks map each other's buffers with
    CUDA IPC at construction (a collective: every rank constructs together).
    Call ``k`` (epoch ``k``) writes the receive buffer of parity ``k & 1`` on
    every rank, so ``decode`` returns a view that keeps its values until the
    call after next: consume it on the same stream before then (the next layer
    of a decode step does) or copy it.  Every rank must make the same sequence
    of calls with the same batch.  Eager only: the epoch is a launch argument,
    so a captured graph would replay a stale one.

    After a device error (``check`` raises, e.g. a peer that never signalled
    within 2 s) the ranks are out of step: build a new instance.
    """

    MAX_RANKS = 64

    def __init__(self, pool, n_q_heads: int, world: int, rank: int, group=None, max_batch: int | None = None):
        super().__init__(pool, n_q_heads, world, rank, group)
        if world > self.MAX_RANKS:
            raise ValueError(f"at most {self.MAX_RANKS} ranks")
        dev = pool.device
        self.max_batch = int(max_batch or pool.max_seqs)
        self.head_dim, self.dtype = pool.head_dim, pool.dtype
        elem = torch.empty((), dtype=pool.dtype).element_size()
        self._out_bytes = (self.max_batch * n_q_heads * self.head_dim * elem + 255) // 256 * 256
        flags_off = 2 * self._out_bytes
        self._buf = torch.zeros(flags_off + 4 * self.MAX_RANKS, dtype=torch.uint8, device=dev)
        self._flags = self._buf[flags_off: flags_off + 4 * world].view(torch.int32)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        lib = _lib.load()
        handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        off = ctypes.c_int64(0)
        _lib.check(lib.snapmind_ipc_export(self._buf.data_ptr(), handle, ctypes.byref(off)), "snapmind_ipc_export")
        torch.cuda.synchronize(dev)  # the zeroed buffer is in place before any peer can write it
        infos: list = [None] * world
        dist.all_gather_object(infos, (handle.raw, int(off.value)), group=group)
        self._handles: list[bytes] = []
        bases = []
        for r, (h, o) in enumerate(infos):
            if r == rank:
                bases.append(self._buf.data_ptr())
            else:
                bases.append(_ipc_open(h, o))
                self._handles.append(h)
        self._out_ptrs = [
            torch.tensor([b + par * self._out_bytes for b in bases], dtype=torch.int64, device=dev)
            for par in (0, 1)
        ]
        self._flag_ptrs = torch.tensor([b + flags_off for b in bases], dtype=torch.int64, device=dev)
        lo, _ = head_range(self.n_kv_total, world, rank)
        self.head_offset = lo * (n_q_heads // self.n_kv_total)
        self.epoch = 0
        dist.barrier(group=group)  # every rank has mapped every buffer

    def decode(self, layer: int, q: torch.Tensor, out: torch.Tensor | None = None, **kw) -> torch.Tensor:
        """q [B, Hq, D] (all heads) -> [B, Hq, D] (all heads, on every rank); a
        view of the receive buffer unless ``out`` is given (then copied there)."""
        b = q.shape[0]
        if b > self.max_batch:
            raise ValueError(f"batch {b} > max_batch {self.max_batch}")
        if b == 0:
            return torch.empty((0, self.n_q_heads, self.head_dim), dtype=self.dtype, device=q.device)
        self.epoch += 1
        par = self.epoch & 1
        q_local = shard_query(q, self.n_kv_total, self.world, self.rank)
        targets = PeerTargets(self._out_ptrs[par], self.world, self.head_offset, self.n_q_heads * self.head_dim,
                              self.head_dim)
        self.pool.decode(layer, q_local, peers=targets, **kw)
        _lib.check(
            _lib.load().snapmind_peer_sync(self._flag_ptrs.data_ptr(), self._flags.data_ptr(), self.world, self.rank,
                                           self.epoch, _lib.PEER_SIGNAL | _lib.PEER_WAIT, self.err.data_ptr(),
                                           self.pool._stream()),
            "snapmind_peer_sync",
        )
        n = b * self.n_q_heads * self.head_dim
        view = self._buf[par * self._out_bytes:].view(self.dtype)[:n].view(b, self.n_q_heads, self.head_dim)
        if out is None:
            return view
        out.copy_(view)
        return out

    def check(self) -> None:
        """Synchronise and raise if a decode or wait of this instance reported a device error."""
        self.pool.check()
        word = int(self.err.item())
        if word:
            _lib.raise_device_error(word, "PeerHeadShardedDecode")

    def close(self) -> None:
        """Unmap the peers' buffers (collective: after every rank's last call)."""
        if self._handles is None:
            return
        torch.cuda.synchronize(self._buf.device)
        dist.barrier(group=self.group)
        for h in self._handles:
            _ipc_release(h)
        self._handles = None
