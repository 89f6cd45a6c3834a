"""Many sequences on a fixed device pool of chunk slots with host-pinned backing.

The batched, device-resident form of the tiered cache
(snapmind/kv_cache/tiered.py): every chunk of ``chunk`` tokens of every
sequence lives in host-pinned backing; a fixed number of chunk slots on the GPU
hold the resident ones.  Placement decisions (new chunks, requested chunks,
least-recently-used eviction, pinning of the sink chunk, the recent window and
the active chunk) are made by the ``snapmind_tiered_plan`` kernel, slot copies
by ``snapmind_tiered_move``; chunk data crosses the host link only as
``cudaMemcpy2DAsync`` copies on a dedicated copy stream:

* requests are copied into fixed inbound staging slots one step ahead
  (``prefetch``), overlapping the previous step's attention;
* a completed chunk is copied by the plan into its sequence's outbound
  staging slot and written back to the backing on the copy stream.

Device layout: ``k``/``v`` are ``[layer][slot][head][chunk][dim]`` — a slot is
one block of the paged layout, so attention runs the paged GQA decode kernel
over ``tables`` (resident slots in chunk order) and ``table_lens``.  Because
the layers are contiguous, block ``slot`` of layer ``l`` is block
``l * total_slots + slot`` of one pool spanning every layer, so one decode
launch serves all layers of a step: row ``l * B + b`` of that launch is
sequence ``b`` of layer ``l`` (its table row shifted by ``l * total_slots``,
its query and output rows at the same index of the contiguous
``[L, B, Hq, D]`` tensors).
"""
from __future__ import annotations

import numpy as np
import torch

from snapmind_b200 import _lib


class TieredKVPool:
    def __init__(
        self,
        n_layers: int,
        n_kv_heads: int,
        head_dim: int,
        batch: int,
        max_tokens: int,
        pool_chunks: int,
        chunk: int = 64,
        sink: int = 4,
        window: int = 1024,
        n_requests: int = 8,
        dtype: torch.dtype = torch.bfloat16,
        device: torch.device | str | None = None,
    ):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        _lib.require_cuda(self.device)
        self.lib = _lib.load()
        self.L, self.H, self.D, self.B = n_layers, n_kv_heads, head_dim, batch
        self.chunk, self.sink, self.window, self.n_requests = chunk, sink, window, n_requests
        self.dtype, self._dcode = dtype, _lib.dtype_code(dtype)
        self.n_slots = pool_chunks
        self.stage_in_base = pool_chunks
        self.stage_out_base = pool_chunks + n_requests
        self.total_slots = pool_chunks + n_requests + batch
        self.max_chunks = (max_tokens + chunk - 1) // chunk
        self.max_plan = n_requests + batch
        shape = (n_layers, self.total_slots, n_kv_heads, chunk, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        esz = self.k.element_size()
        self.slot_bytes = n_kv_heads * chunk * head_dim * esz
        self.layer_stride_bytes = self.total_slots * self.slot_bytes
        i32 = dict(dtype=torch.int32, device=self.device)
        self.slot_owner = torch.full((pool_chunks,), -1, **i32)
        self.slot_last = torch.zeros(pool_chunks, **i32)
        self.chunk_slot = torch.full((batch, self.max_chunks), -1, **i32)
        self.seq_lens = torch.zeros(batch, **i32)
        self.tables = torch.zeros((batch, self.max_chunks), **i32)
        self.table_lens = torch.zeros(batch, **i32)
        self.plan = torch.zeros((self.max_plan, 2), **i32)
        self.plan_count = torch.zeros(1, **i32)
        self.err = torch.zeros(1, **i32)
        # host backing: per (sequence, chunk) K rows of every layer then V rows
        self.backing = torch.empty((batch, self.max_chunks, 2, n_layers, n_kv_heads, chunk, head_dim), dtype=dtype,
                                   pin_memory=True)
        self.chunk_host_bytes = 2 * n_layers * self.slot_bytes
        self.copy_stream = torch.cuda.Stream(self.device)
        self._staging_free = torch.cuda.Event()
        self._staged = torch.cuda.Event()
        self._snap = [torch.empty((batch, self.max_chunks), dtype=torch.int32, pin_memory=True) for _ in range(3)]
        self._snap_ev = [torch.cuda.Event() for _ in range(3)]
        self.host_lens = np.zeros(batch, np.int64)
        self.step_idx = 0
        self._workspace = _lib.DecodeWorkspace(self.device)
        # one decode launch for all layers: per-layer block offsets of the shared tables
        self._layer_offsets = (torch.arange(n_layers, dtype=torch.int32, device=self.device)
                               * self.total_slots).view(n_layers, 1, 1)
        self._tables_all = torch.zeros((n_layers, batch, self.max_chunks), **i32)
        self._lens_all = torch.zeros((n_layers, batch), **i32)
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    # ------------------------------------------------------------ host <-> device
    def _stream(self, s=None) -> int:
        return (s or torch.cuda.current_stream(self.device)).cuda_stream

    def _copy_chunk(self, to_device: bool, slot: int, b: int, c: int, stream) -> None:
        """K and V rows of every layer of chunk (b, c) between its backing and `slot`."""
        for kv, pool in ((0, self.k), (1, self.v)):
            dev = pool.data_ptr() + slot * self.slot_bytes
            host = self.backing[b, c, kv].data_ptr()
            if to_device:
                rc = self.lib.snapmind_copy_2d(dev, self.layer_stride_bytes, host, self.slot_bytes, self.slot_bytes,
                                               self.L, self._stream(stream))
                self.h2d_bytes += self.L * self.slot_bytes
            else:
                rc = self.lib.snapmind_copy_2d(host, self.slot_bytes, dev, self.layer_stride_bytes, self.slot_bytes,
                                               self.L, self._stream(stream))
                self.d2h_bytes += self.L * self.slot_bytes
            _lib.check(rc, "TieredKVPool copy")

    def fill_backing(self, seed: int, lens: np.ndarray) -> None:
        """Seeded N(0,1) K/V for every chunk below lens[b] (generated on the GPU, copied down)."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        per = self.backing[0].numel() // self.max_chunks  # elements per chunk
        for b in range(self.B):
            n = (int(lens[b]) + self.chunk - 1) // self.chunk
            if n:
                buf = torch.randn((n, per), generator=g, device=self.device).to(self.dtype)
                self.backing[b, :n].view(n, per).copy_(buf)
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------ state
    def install(self, lens: np.ndarray, resident: list[list[int]]) -> None:
        """Set lengths and place the listed chunks of each sequence in slots 0, 1, ... (in order)."""
        owner = np.full(self.n_slots, -1, np.int64)
        cslot = np.full((self.B, self.max_chunks), -1, np.int64)
        s = 0
        for b, chunks in enumerate(resident):
            for c in chunks:
                if s >= self.n_slots:
                    raise RuntimeError("resident set larger than the pool")
                owner[s] = (b << 16) | c
                cslot[b, c] = s
                s += 1
        self.slot_owner.copy_(torch.from_numpy(owner.astype(np.int32)))
        self.slot_last.zero_()
        self.chunk_slot.copy_(torch.from_numpy(cslot.astype(np.int32)))
        self.seq_lens.copy_(torch.from_numpy(np.asarray(lens, np.int32)))
        self.host_lens = np.asarray(lens, np.int64).copy()
        for b, chunks in enumerate(resident):
            for c in chunks:
                self._copy_chunk(True, int(cslot[b, c]), b, c, torch.cuda.current_stream(self.device))
        self._plan(0, [])  # rebuild tables (no growth, no requests)
        self.step_idx = 0
        torch.cuda.synchronize(self.device)
        # every residency snapshot starts as the installed map: the snapshot read at
        # step 2 is the one of step 0, which no step writes
        installed = self.chunk_slot.cpu()
        for snap, ev in zip(self._snap, self._snap_ev):
            snap.copy_(installed)
            ev.record(torch.cuda.current_stream(self.device))

    def _check_requests(self, requests: list[tuple[int, int]]) -> None:
        if len(requests) > self.n_requests:
            raise ValueError(f"TieredKVPool: {len(requests)} requests exceed the {self.n_requests} staging slots")

    def check(self) -> None:
        word = int(self.err.item())
        if word:
            self.err.zero_()
            _lib.raise_device_error(word, "TieredKVPool")

    # ------------------------------------------------------------ one step
    def _plan(self, n_new: int, requests: list[tuple[int, int]]) -> None:
        n = len(requests)
        arr = _lib.ctypes.c_int32 * max(1, n)
        rs = arr(*[r[0] for r in requests]) if n else arr()
        rc_ = arr(*[r[1] for r in requests]) if n else arr()
        status = self.lib.snapmind_tiered_plan(
            self.slot_owner.data_ptr(), self.slot_last.data_ptr(), self.chunk_slot.data_ptr(),
            self.seq_lens.data_ptr(), self.tables.data_ptr(), self.table_lens.data_ptr(),
            self.plan.data_ptr(), self.plan_count.data_ptr(), self.B, self.max_chunks, self.n_slots,
            self.chunk, self.sink, self.window, self.step_idx, n_new, self.stage_in_base, self.stage_out_base,
            self.max_plan, rs, rc_, n, self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "TieredKVPool.plan")

    def prefetch(self, requests: list[tuple[int, int]]) -> None:
        """Copy the next step's requested chunks into the inbound staging slots (copy stream)."""
        self._check_requests(requests)
        cs = self.copy_stream
        cs.wait_event(self._staging_free)
        for i, (b, c) in enumerate(requests):
            self._copy_chunk(True, self.stage_in_base + i, b, c, cs)
        self._staged.record(cs)

    def snapshot(self, age: int = 2) -> np.ndarray | None:
        """chunk -> slot map as of ``age`` steps ago (None before that many steps)."""
        if self.step_idx < age:
            return None
        i = (self.step_idx - age) % 3
        self._snap_ev[i].synchronize()
        return self._snap[i].numpy()

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, out: torch.Tensor,
             requests: list[tuple[int, int]], next_requests: list[tuple[int, int]] | None = None,
             split_tokens: int = 0) -> None:
        """One decode step: q [L, B, Hq, D], k_new/v_new [L, B, H, D], out [L, B, Hq, D].

        ``requests`` must have been passed to ``prefetch`` (or as ``next_requests``
        of the previous step); ``next_requests`` are prefetched after this
        step's slot moves so their copies overlap this step's attention.
        """
        self._check_requests(requests)
        if next_requests:
            self._check_requests(next_requests)
        main = torch.cuda.current_stream(self.device)
        self.step_idx += 1
        if requests:
            main.wait_event(self._staged)
        old = self.host_lens.copy()
        self._plan(1, requests)
        status = self.lib.snapmind_tiered_move(self.k.data_ptr(), self.v.data_ptr(), self.layer_stride_bytes,
                                               self.slot_bytes, self.L, self.plan.data_ptr(),
                                               self.plan_count.data_ptr(), self.max_plan, self._stream())
        _lib.check(status, "TieredKVPool.move")
        self._staging_free.record(main)
        self.host_lens += 1
        # write-backs of completed chunks, the residency snapshot, then the next prefetch
        cs = self.copy_stream
        cs.wait_event(self._staging_free)
        for b in np.nonzero((old > 0) & (old % self.chunk == 0))[0]:
            self._copy_chunk(False, self.stage_out_base + int(b), int(b), int(old[b] // self.chunk - 1), cs)
        si = self.step_idx % 3
        with torch.cuda.stream(cs):
            self._snap[si].copy_(self.chunk_slot, non_blocking=True)
        self._snap_ev[si].record(cs)
        if next_requests:
            self.prefetch(next_requests)
        # append the new token of every layer, then attention per layer
        st = k_new.stride()
        status = self.lib.snapmind_kv_append(
            self.k.data_ptr(), self.v.data_ptr(), self._dcode, self.layer_stride_bytes // self.k.element_size(),
            k_new.data_ptr(), v_new.data_ptr(), _lib.dtype_code(k_new.dtype), st[0], st[1], st[2], 0,
            self.chunk_slot.data_ptr(), self.max_chunks, 0, self.max_chunks, self.seq_lens.data_ptr(), -1,
            self.L, self.B, 1, self.H, self.D, self.chunk, self.total_slots, self.err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "TieredKVPool.append")
        max_len = self._resident_bound() * self.chunk
        one_launch = q.is_contiguous() and out.is_contiguous()
        rows = self.B * self.L if one_launch else self.B
        # split plan sized for the launch's rows and the average resident length (the pool
        # shared by the batch)
        split = split_tokens or self.lib.snapmind_paged_gqa_decode_split_tokens(
            rows, self.H, max(self.chunk, 2 * self.n_slots * self.chunk // self.B), self.chunk)
        need = self.lib.snapmind_paged_gqa_decode_workspace_bytes(rows, q.shape[2], self.H, self.D, max_len, split)
        ws = self._workspace.get(rows, self.H, need)
        if one_launch:
            # every layer in one launch: row l * B + b = sequence b of layer l
            torch.add(self.tables.unsqueeze(0), self._layer_offsets, out=self._tables_all)
            self._lens_all.copy_(self.table_lens.unsqueeze(0).expand(self.L, self.B))
            status = self.lib.snapmind_paged_gqa_decode(
                q.data_ptr(), q.stride(1), q.stride(2), self.k.data_ptr(), self.v.data_ptr(), self._dcode,
                self._tables_all.data_ptr(), self.max_chunks, self.max_chunks, self._lens_all.data_ptr(),
                out.data_ptr(), out.stride(1), out.stride(2), float(self.D ** -0.5), rows, q.shape[2], self.H,
                self.D, self.chunk, self.L * self.total_slots, max_len, split, 0, ws.data_ptr(), ws.numel(),
                self.err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "TieredKVPool.decode")
            return
        for layer in range(self.L):
            qs, os_ = q[layer], out[layer]
            status = self.lib.snapmind_paged_gqa_decode(
                qs.data_ptr(), qs.stride(0), qs.stride(1), self.k[layer].data_ptr(), self.v[layer].data_ptr(),
                self._dcode, self.tables.data_ptr(), self.max_chunks, self.max_chunks, self.table_lens.data_ptr(),
                os_.data_ptr(), os_.stride(0), os_.stride(1), float(self.D ** -0.5), self.B, qs.shape[1], self.H,
                self.D, self.chunk, self.total_slots, max_len, split, 0, ws.data_ptr(), ws.numel(),
                self.err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "TieredKVPool.decode")

    def _resident_bound(self) -> int:
        """An upper bound on any sequence's resident chunks at this step's decode:
        the largest count in the residency snapshot of two steps ago plus what
        three steps can add (per step at most the requested chunks and one new
        chunk per sequence), capped at the pool's slots.  It sizes the decode's
        split plan; without a snapshot yet, every slot."""
        cap = self.n_slots
        snap = self.snapshot(2)
        if snap is None:
            return cap
        most = int((snap >= 0).sum(axis=1).max()) if snap.size else 0
        return max(1, min(cap, most + 3 * (self.n_requests + 1)))

    def pick_requests(self, rng: np.random.RandomState, n: int, exclude: set | None = None) -> list[tuple[int, int]]:
        """n seeded-random chunks that were cold two steps ago (completed, unpinned, not recently requested)."""
        snap = self.snapshot(2)
        exclude = exclude or set()
        out: list[tuple[int, int]] = []
        tries = 0
        while len(out) < n and tries < 100 * n:
            tries += 1
            b = int(rng.randint(self.B))
            length = int(self.host_lens[b])
            done = length // self.chunk  # completed chunks
            lo = 1 if self.sink > 0 else 0
            hi = min(done, max(0, (length - self.window) // self.chunk))  # chunks entirely before the window
            if hi <= lo:
                continue
            c = int(rng.randint(lo, hi))
            if (b, c) in exclude or (b, c) in out:
                continue
            if snap is not None and snap[b, c] >= 0:
                continue
            out.append((b, c))
        return out
