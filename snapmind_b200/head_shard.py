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

Both offer ``decode_step``: every layer of one decode step (``q [L, B, Hq, D]``)
in one decode launch (``PagedKVPool.decode_layers``) with one exchange for the
whole step instead of one per layer -- one all-gather of ``[L, B, Hq/N, D]``
for the NCCL form, and for the peer-store form every layer's rows stored into
that layer's slice of an ``[L, B, Hq, D]`` receive region, followed by a
single epoch signal and wait.
It suits callers whose consumer of the outputs runs after the whole step; a
model layer that needs layer l's heads before layer l + 1 uses ``decode``.
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

    def decode_step(self, q_layers: torch.Tensor, out: torch.Tensor | None = None, **kw) -> torch.Tensor:
        """Layers 0 .. L-1 of one step: q [L, B, Hq, D] -> [L, B, Hq, D], one all-gather."""
        n_l, b, n_q, d = q_layers.shape
        hl = n_q // self.world
        local = torch.empty((n_l, b, hl, d), dtype=q_layers.dtype, device=q_layers.device)
        group = n_q // self.n_kv_total
        lo, hi = head_range(self.n_kv_total, self.world, self.rank)
        q_local = q_layers[:, :, lo * group: hi * group]
        if hasattr(self.pool, "decode_layers") and q_local.stride(0) == b * q_local.stride(1):
            self.pool.decode_layers(q_local, out=local, **kw)  # every layer in one launch
        else:
            for layer in range(n_l):
                self.pool.decode(layer, q_local[layer], out=local[layer], **kw)
        gathered = torch.empty((self.world, n_l, b, hl, d), dtype=local.dtype, device=local.device)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(gathered, local, group=self.group)
        else:
            dist.all_gather(list(gathered.unbind(0)), local, group=self.group)
        if out is None:
            out = torch.empty((n_l, b, n_q, d), dtype=local.dtype, device=local.device)
        out.view(n_l, b, self.world, hl, d).copy_(gathered.permute(1, 2, 0, 3, 4))
        return out


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

    Each rank owns one device buffer holding two receive regions of
    ``n_layers`` ``[max_batch, Hq, D]`` slices and an int32 flag per rank; the
    ranks map each other's buffers with CUDA IPC at construction (a collective:
    every rank constructs together).  Call ``k`` (epoch ``k``, one ``decode`` or
    one ``decode_step``) writes the region of parity ``k & 1`` on every rank, so
    the returned view keeps its values until the call after next: consume it on
    the same stream before then (the next layer of a decode step does) or copy
    it.  Every rank must make the same sequence
    of calls with the same batch.  Eager only: the epoch is a launch argument,
    so a captured graph would replay a stale one.

    After a device error (``check`` raises, e.g. a peer that never signalled
    within 2 s) the ranks are out of step: build a new instance.
    """

    MAX_RANKS = 64

    def __init__(self, pool, n_q_heads: int, world: int, rank: int, group=None, max_batch: int | None = None,
                 n_layers: int = 1):
        super().__init__(pool, n_q_heads, world, rank, group)
        if world > self.MAX_RANKS:
            raise ValueError(f"at most {self.MAX_RANKS} ranks")
        dev = pool.device
        self.max_batch = int(max_batch or pool.max_seqs)
        self.n_layers = int(n_layers)
        self.head_dim, self.dtype = pool.head_dim, pool.dtype
        elem = torch.empty((), dtype=pool.dtype).element_size()
        self._elem = elem
        self._out_bytes = (self.max_batch * n_q_heads * self.head_dim * elem + 255) // 256 * 256  # one slice
        self._region_bytes = self.n_layers * self._out_bytes  # one parity
        flags_off = 2 * self._region_bytes
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
        # [parity][layer][rank]: the destination of each (parity, layer slice) on every rank
        self._slice_ptrs = torch.tensor(
            [[[b + par * self._region_bytes + layer * self._out_bytes for b in bases]
              for layer in range(self.n_layers)] for par in (0, 1)],
            dtype=torch.int64, device=dev)
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
        self._decode_into(layer, q, par, 0, **kw)
        self._sync()
        view = self._region(par, 1, b)[0]
        if out is None:
            return view
        out.copy_(view)
        return out

    def decode_step(self, q_layers: torch.Tensor, out: torch.Tensor | None = None, **kw) -> torch.Tensor:
        """Layers 0 .. L-1 of one step (q [L, B, Hq, D]) with a single epoch signal and
        wait after the last layer; returns a view [L, B, Hq, D] of the receive region
        unless ``out`` is given (then copied there)."""
        n_l, b = q_layers.shape[:2]
        if n_l > self.n_layers:
            raise ValueError(f"{n_l} layers > the {self.n_layers} receive slices (n_layers)")
        if b > self.max_batch:
            raise ValueError(f"batch {b} > max_batch {self.max_batch}")
        self.epoch += 1
        par = self.epoch & 1
        group = self.n_q_heads // self.n_kv_total
        lo, hi = head_range(self.n_kv_total, self.world, self.rank)
        q_local = q_layers[:, :, lo * group: hi * group]
        if b == self.max_batch and self._out_bytes == b * self.n_q_heads * self.head_dim * self._elem and \
                q_local.stride(0) == b * q_local.stride(1):
            # every layer in one launch: row l * B + b lands in layer l's slice of each rank's region
            targets = PeerTargets(self._slice_ptrs[par, 0], self.world, self.head_offset,
                                  self.n_q_heads * self.head_dim, self.head_dim)
            self.pool.decode_layers(q_local, peers=targets, **kw)
        else:
            for layer in range(n_l):
                self._decode_into(layer, q_layers[layer], par, layer, **kw)
        self._sync()
        view = self._region(par, n_l, b)
        if out is None:
            return view
        out.copy_(view)
        return out

    def _decode_into(self, layer: int, q: torch.Tensor, par: int, slot: int, **kw) -> None:
        q_local = shard_query(q, self.n_kv_total, self.world, self.rank)
        targets = PeerTargets(self._slice_ptrs[par, slot], self.world, self.head_offset,
                              self.n_q_heads * self.head_dim, self.head_dim)
        self.pool.decode(layer, q_local, peers=targets, **kw)

    def _sync(self) -> None:
        _lib.check(
            _lib.load().snapmind_peer_sync(self._flag_ptrs.data_ptr(), self._flags.data_ptr(), self.world, self.rank,
                                           self.epoch, _lib.PEER_SIGNAL | _lib.PEER_WAIT, self.err.data_ptr(),
                                           self.pool._stream()),
            "snapmind_peer_sync",
        )

    def _region(self, par: int, n_l: int, b: int) -> torch.Tensor:
        """[n_l, b, Hq, D] view of the first slices of the parity-``par`` region."""
        flat = self._buf[par * self._region_bytes:].view(self.dtype)
        row = self.n_q_heads * self.head_dim
        return flat.as_strided((n_l, b, self.n_q_heads, self.head_dim),
                               (self._out_bytes // self._elem, row, self.head_dim, 1))

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
