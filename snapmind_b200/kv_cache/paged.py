"""PagedKVCache on the B200: device block pool, host block bookkeeping.

Drop-in for ``snapmind.kv_cache.paged.PagedKVCache`` (snapmind/kv_cache/paged.py:9-145),
registered under the same key ``"paged"`` in this package's ``KV_CACHE``.

What stays on the host (bookkeeping, exactly as the reference does it, so block
tables are bit-identical): the free-block ``set`` and its ``pop()`` order, the
per-layer block-table lists sharing that one set, the per-layer slot counts,
and the evict plan.  What runs on the GPU (hand-written sm_100a kernels through
the C ABI): every byte of K/V — the append of ``store``, the tile gather of
``fetch``/``layer_dicts`` and the compaction copy of ``evict``.

Differences a caller can see: the pool and the tensors ``fetch`` returns live on
the CUDA device; the pool dtype is ``dtype`` (default float32, the reference's
default).  Device block tables are mirrored in an int32 tensor updated when a
table grows.  ``layer_dicts`` returns per-layer views (:class:`PagedLayerView`)
instead of detached copies: they read like the reference's dicts, and what an
attention layer assigns to them is written into the pool — the reference's
models grow copies with ``torch.cat`` and never write its pool
(snapmind/engine/generate.py:88-90, snapmind/layers/attention/gqa.py:62-67).
``attend`` runs paged GQA attention for the newest tokens of a layer straight
from the pool.
"""
from __future__ import annotations

import ctypes
from collections.abc import MutableMapping

import torch

from snapmind_b200 import _lib
from snapmind_b200.kv_cache.base import KVCacheABC
from snapmind_b200.registry import KV_CACHE

_KERNEL_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _default_device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("snapmind_b200 PagedKVCache needs a CUDA device")
    return torch.device("cuda", torch.cuda.current_device())


@KV_CACHE.register("paged")
class PagedKVCache(KVCacheABC):
    def __init__(
        self,
        max_seq_len: int,
        n_layers: int,
        n_heads: int,
        head_dim: int,
        block_size: int = 16,
        max_blocks: int | None = None,
        *,
        dtype: torch.dtype = torch.float32,
        device: torch.device | str | None = None,
    ):
        self.n_layers = n_layers
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.block_size = block_size
        # snapmind/kv_cache/paged.py:24-25
        max_blocks = max_blocks or (max_seq_len + block_size - 1) // block_size
        self.max_blocks = max_blocks
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else _default_device()
        _lib.require_cuda(self.device)
        _lib.dtype_code(dtype)
        _lib.load()

        # pool[block][head][slot][dim]: a (block, head) tile is contiguous
        shape = (max_blocks, n_heads, block_size, head_dim)
        self._k_buffer = torch.zeros(shape, dtype=dtype, device=self.device)
        self._v_buffer = torch.zeros(shape, dtype=dtype, device=self.device)
        self._free_blocks = set(range(max_blocks))
        self._block_tables: list[list[int]] = [[] for _ in range(n_layers)]
        self._slot_counts: list[int] = [0] * n_layers
        self._tables_dev = torch.zeros((n_layers, max_blocks), dtype=torch.int32, device=self.device)
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._version = 0  # bumped by every change of the cached contents
        self._ladder: torch.Tensor | None = None  # int32 [1, 2, ..., max_blocks * block_size]
        self._workspace = _lib.DecodeWorkspace(self.device)
        # device-counter steps (begin_device_steps): slot of the next token, and length after it
        self._dev_len: torch.Tensor | None = None
        self._dev_len_p1: torch.Tensor | None = None
        self._dev_steps = 0
        self._dev_capacity = 0

    # ------------------------------------------------------------------ helpers
    def _stream(self) -> int:
        return _lib.stream_handle(self.device)

    def _sync_table(self, layer_idx: int, old_len: int) -> None:
        bt = self._block_tables[layer_idx]
        if len(bt) > old_len:
            new = torch.tensor(bt[old_len:], dtype=torch.int32)
            self._tables_dev[layer_idx, old_len : len(bt)].copy_(new, non_blocking=False)

    def _as_input(self, t: torch.Tensor) -> torch.Tensor:
        if t.device != self.device:
            t = t.to(self.device)
        if t.dtype not in _KERNEL_DTYPES:
            t = t.to(self.dtype)
        if t.stride(-1) != 1:
            t = t.contiguous()
        return t

    def check_device_errors(self) -> None:
        """Synchronise and raise if any kernel of this cache flagged an error."""
        word = int(self._err.item())
        if word:
            self._err.zero_()
            _lib.raise_device_error(word, "PagedKVCache")

    # --------------------------------------------------------------------- API
    def store(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, seq_pos: int) -> None:
        """Append ``key[0, :, t, :]`` / ``value[0, :, t, :]`` for every t.

        Mirrors snapmind/kv_cache/paged.py:34-54: ``seq_pos`` is ignored, tokens
        go to the next free slots of the layer, blocks come from ``set.pop()``;
        on exhaustion the tokens that already had a block are written, the
        blocks taken so far stay in the table, the slot count is unchanged and
        ``RuntimeError("PagedKVCache: out of blocks")`` is raised.
        """
        num_tokens = key.shape[-2]
        slot_start = self._slot_counts[layer_idx]
        bt = self._block_tables[layer_idx]
        old_len = len(bt)
        failed = False
        if num_tokens > 0:
            last_block = (slot_start + num_tokens - 1) // self.block_size
            while len(bt) <= last_block:
                if not self._free_blocks:
                    failed = True
                    break
                bt.append(self._free_blocks.pop())
        writable = min(num_tokens, max(0, len(bt) * self.block_size - slot_start))
        self._sync_table(layer_idx, old_len)
        if writable > 0:
            if key.shape[1] != self.n_heads or key.shape[-1] != self.head_dim:
                raise RuntimeError(
                    f"PagedKVCache.store: expected (1, {self.n_heads}, T, {self.head_dim}) rows, "
                    f"got {tuple(key.shape)}"
                )
            k = self._as_input(key[0])  # (H, T, D)
            v = self._as_input(value[0])
            if v.stride() != k.stride() or v.dtype != k.dtype:
                k, v = k.contiguous(), v.to(k.dtype).contiguous()
            status = _lib.load().snapmind_kv_append(
                self._k_buffer.data_ptr(), self._v_buffer.data_ptr(), _lib.dtype_code(self.dtype), 0,
                k.data_ptr(), v.data_ptr(), _lib.dtype_code(k.dtype),
                0, 0, k.stride(0), k.stride(1),
                self._tables_dev[layer_idx].data_ptr(), 0, 0, self.max_blocks,
                None, slot_start,
                1, 1, writable, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
                self._err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "PagedKVCache.store")
        self._version += 1
        if failed:
            raise RuntimeError(_lib.OUT_OF_BLOCKS_MSG)
        self._slot_counts[layer_idx] = slot_start + num_tokens

    def fetch(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Return ``(k, v)`` of shape ``(1, H, T, D)`` (snapmind/kv_cache/paged.py:56-78).

        An empty table returns two ``(0, H, D)`` tensors, as the reference does.
        """
        bt = self._block_tables[layer_idx]
        if not bt:
            return (
                torch.empty(0, self.n_heads, self.head_dim, dtype=self.dtype, device=self.device),
                torch.empty(0, self.n_heads, self.head_dim, dtype=self.dtype, device=self.device),
            )
        num_slots = self._slot_counts[layer_idx]
        if num_slots == 0:
            # the reference concatenates an empty list here
            raise RuntimeError("torch.cat(): expected a non-empty list of Tensors")
        k = torch.empty((1, self.n_heads, num_slots, self.head_dim), dtype=self.dtype, device=self.device)
        v = torch.empty_like(k)
        status = _lib.load().snapmind_kv_gather(
            self._k_buffer.data_ptr(), self._v_buffer.data_ptr(), _lib.dtype_code(self.dtype), 0,
            k.data_ptr(), v.data_ptr(), 0, k.numel(),
            self._tables_dev[layer_idx].data_ptr(), 0, 0, self.max_blocks,
            None, num_slots,
            1, 1, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
            self._err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVCache.fetch")
        return k, v

    def _copy_rows(self, rows: list[tuple[int, int, int, int]]) -> None:
        """Device copy of (src_block, src_row, dst_block, dst_row) rows, in
        ascending chunks of at most 64 rows, each chunk read before written."""
        lib = _lib.load()
        arr = ctypes.c_int32 * 64
        for c in range(0, len(rows), 64):
            chunk = rows[c : c + 64]
            sb, sr, db, dr = (arr(*[r[i] for r in chunk]) for i in range(4))
            status = lib.snapmind_kv_copy_slots(
                self._k_buffer.data_ptr(), self._v_buffer.data_ptr(), _lib.dtype_code(self.dtype),
                sb, sr, db, dr, len(chunk), self.n_heads, self.head_dim, self.block_size,
                self.max_blocks, self._err.data_ptr(), self._stream(),
            )  # fmt: skip
            _lib.check(status, "PagedKVCache.evict")

    def evict(self, tokens_to_keep: int) -> None:
        """Keep the newest ``tokens_to_keep`` tokens per layer.

        Mirrors snapmind/kv_cache/paged.py:80-116 step by step, including its
        limits: when the start is not block aligned the kept tokens are packed
        into the first kept block, which the reference can only do when they fit
        in it — otherwise its slice assignment raises ``RuntimeError`` after the
        freed blocks were returned and the earlier packing steps were written;
        this implementation reproduces that state and raises the same type.
        """
        bs = self.block_size
        self._version += 1
        for layer_idx in range(self.n_layers):
            total = self._slot_counts[layer_idx]
            if total <= tokens_to_keep:
                continue
            start_slot = total - tokens_to_keep
            start_block = start_slot // bs
            offset_in_block = start_slot % bs
            bt = self._block_tables[layer_idx]
            blocks_needed = (offset_in_block + tokens_to_keep + bs - 1) // bs
            kept_blocks = bt[start_block : start_block + blocks_needed]
            freed_blocks = bt[:start_block] + bt[start_block + blocks_needed :]
            for b in freed_blocks:
                self._free_blocks.add(b)

            if offset_in_block > 0 and kept_blocks:
                first = kept_blocks[0]
                remaining = tokens_to_keep
                src_off = offset_in_block
                dst_off = 0
                rows: list[tuple[int, int, int, int]] = []
                error: str | None = None
                for b in kept_blocks:
                    take = min(bs - src_off, remaining)
                    dst_len = max(0, min(bs, dst_off + take) - min(bs, dst_off))
                    if dst_len != take:
                        error = (
                            f"The expanded size of the tensor ({dst_len}) must match the existing "
                            f"size ({take}) at non-singleton dimension 0."
                        )
                        break
                    rows.extend((b, src_off + i, first, dst_off + i) for i in range(take))
                    dst_off += take
                    remaining -= take
                    src_off = 0
                self._copy_rows(rows)
                if error is not None:
                    raise RuntimeError(error)
                needed = (dst_off + bs - 1) // bs
                for b in kept_blocks[needed:]:
                    self._free_blocks.add(b)
                kept_blocks = kept_blocks[:needed]

            self._block_tables[layer_idx] = kept_blocks
            if kept_blocks:
                self._tables_dev[layer_idx, : len(kept_blocks)].copy_(
                    torch.tensor(kept_blocks, dtype=torch.int32)
                )
            self._slot_counts[layer_idx] = tokens_to_keep

    def reset(self) -> None:
        self._k_buffer.zero_()
        self._v_buffer.zero_()
        self._free_blocks = set(range(self.max_blocks))
        self._block_tables = [[] for _ in range(self.n_layers)]
        self._slot_counts = [0] * self.n_layers
        self._tables_dev.zero_()
        self._version += 1

    def memory_usage(self) -> dict:
        total_bytes = self._k_buffer.numel() * self._k_buffer.element_size()
        total_bytes += self._v_buffer.numel() * self._v_buffer.element_size()
        return {
            "num_tokens": sum(self._slot_counts),
            "total_bytes": total_bytes,
            "used_blocks": sum(len(bt) for bt in self._block_tables),
            "max_blocks": self.max_blocks,
        }

    def layer_dicts(self) -> dict[int, "PagedLayerView"]:
        """One :class:`PagedLayerView` per layer (snapmind/kv_cache/paged.py:137-145
        returns ``{"k": None, "v": None}`` or fetched copies; the views read the
        same and write assignments through to the pool)."""
        return {i: PagedLayerView(self, i) for i in range(self.n_layers)}

    def num_tokens(self, layer_idx: int) -> int:
        return self._slot_counts[layer_idx]

    def _lens_ladder(self) -> torch.Tensor:
        if self._ladder is None:
            n = self.max_blocks * self.block_size
            self._ladder = torch.arange(1, n + 1, dtype=torch.int32, device=self.device)
        return self._ladder

    def attend(self, layer_idx: int, q: torch.Tensor, scale: float | None = None, causal: bool = True,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """Paged GQA attention of the queries of the newest ``T`` tokens of a layer.

        ``q``: ``(1, Hq, T, D)`` in the pool dtype, ``Hq`` a multiple of the
        cache's kv heads.  With ``causal`` query ``t`` attends to the first
        ``n - T + t + 1`` cached tokens (``n`` = tokens in the layer), the
        causal mask of snapmind/layers/attention/sdpa.py ``create_causal_mask``
        shifted to the end of the cache; otherwise every query attends to all
        ``n`` tokens (the reference's decode with ``mask=None``).  Every query
        is one row of the paged decode kernel: all rows share this layer's
        block table (row stride 0), and the causal lengths are read from a
        constant device array ``1, 2, 3, ...``, so no lengths are copied.
        Returns ``(1, Hq, T, D)``.
        """
        if q.dim() != 4 or q.shape[0] != 1 or q.shape[-1] != self.head_dim:
            raise ValueError(f"attend: expected q of shape (1, Hq, T, {self.head_dim}), got {tuple(q.shape)}")
        if q.dtype != self.dtype:
            raise TypeError(f"attend: q dtype {q.dtype} != cache dtype {self.dtype}")
        n_q, n_t = q.shape[1], q.shape[2]
        n = self._slot_counts[layer_idx]
        if n_t > n:
            raise ValueError(f"attend: {n_t} queries but only {n} cached tokens in layer {layer_idx}")
        if q.stride(-1) != 1:
            q = q.contiguous()
        if out is None:
            out = torch.empty((1, n_q, n_t, self.head_dim), dtype=self.dtype, device=self.device)
        if n_t == 0:
            return out
        if causal:
            lens = self._lens_ladder()
            lens_ptr = lens.data_ptr() + 4 * (n - n_t)
        else:
            lens = torch.full((n_t,), n, dtype=torch.int32, device=self.device)
            lens_ptr = lens.data_ptr()
        scale = self.head_dim ** -0.5 if scale is None else scale
        lib = _lib.load()
        split = lib.snapmind_paged_gqa_decode_split_tokens(n_t, self.n_heads, n, self.block_size)
        need = lib.snapmind_paged_gqa_decode_workspace_bytes(n_t, n_q, self.n_heads, self.head_dim, n, split)
        ws = self._workspace.get(n_t, self.n_heads, need)
        status = lib.snapmind_paged_gqa_decode(
            q.data_ptr(), q.stride(2), q.stride(1),
            self._k_buffer.data_ptr(), self._v_buffer.data_ptr(), _lib.dtype_code(self.dtype),
            self._tables_dev[layer_idx].data_ptr(), 0, self.max_blocks, lens_ptr,
            out.data_ptr(), out.stride(2), out.stride(1),
            float(scale), n_t, n_q, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
            n, split, 0, ws.data_ptr(), ws.numel(), self._err.data_ptr(),
            self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVCache.attend")
        return out

    # ------------------------------------------- device-counter steps (CUDA graphs)
    @property
    def device_steps_active(self) -> bool:
        return self._dev_len is not None

    def begin_device_steps(self, n_steps: int) -> None:
        """Prepare ``n_steps`` one-token steps whose slot and length live in device
        counters, so that a whole decode step can be captured in a CUDA graph and
        replayed without host work.

        Every layer must hold the same number of tokens.  The blocks those steps
        need are taken now, in the order the reference's per-token stores would
        take them (step by step, layer by layer: snapmind/kv_cache/paged.py:43-47),
        so the block tables end up as an eager run's; the steps must then all be
        run before ``end_device_steps``.
        """
        if self._dev_len is not None:
            raise RuntimeError("PagedKVCache: device steps already active")
        counts = set(self._slot_counts)
        if len(counts) != 1:
            raise ValueError("PagedKVCache.begin_device_steps: every layer must hold the same number of tokens")
        n0 = counts.pop()
        if n_steps <= 0:
            raise ValueError("PagedKVCache.begin_device_steps: n_steps must be positive")
        old = [len(bt) for bt in self._block_tables]
        for step in range(n_steps):
            blk = (n0 + step) // self.block_size
            for layer_idx in range(self.n_layers):
                bt = self._block_tables[layer_idx]
                while len(bt) <= blk:
                    if not self._free_blocks:
                        for li in range(self.n_layers):
                            self._sync_table(li, old[li])
                        raise RuntimeError(_lib.OUT_OF_BLOCKS_MSG)
                    bt.append(self._free_blocks.pop())
        for layer_idx in range(self.n_layers):
            self._sync_table(layer_idx, old[layer_idx])
        self._dev_len = torch.full((1,), n0, dtype=torch.int32, device=self.device)
        self._dev_len_p1 = torch.full((1,), n0 + 1, dtype=torch.int32, device=self.device)
        self._dev_steps = n_steps
        self._dev_capacity = n0 + n_steps

    def store_device(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append one token (``key``/``value`` ``(1, H, 1, D)``) at the slot held by the
        device counter.  No host work, no sync: capturable in a CUDA graph."""
        k = self._as_input(key[0])
        v = self._as_input(value[0])
        if v.stride() != k.stride() or v.dtype != k.dtype:
            k, v = k.contiguous(), v.to(k.dtype).contiguous()
        status = _lib.load().snapmind_kv_append(
            self._k_buffer.data_ptr(), self._v_buffer.data_ptr(), _lib.dtype_code(self.dtype), 0,
            k.data_ptr(), v.data_ptr(), _lib.dtype_code(k.dtype),
            0, 0, k.stride(0), k.stride(1),
            self._tables_dev[layer_idx].data_ptr(), 0, 0, self.max_blocks,
            self._dev_len.data_ptr(), 0,
            1, 1, 1, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
            self._err.data_ptr(), self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVCache.store_device")

    def attend_device(self, layer_idx: int, q: torch.Tensor, scale: float | None = None) -> torch.Tensor:
        """Decode attention of one query ``(1, Hq, 1, D)`` over the tokens up to and
        including the device counter's slot; the split plan is fixed by the
        capacity reserved in ``begin_device_steps``."""
        if q.dtype != self.dtype:
            raise TypeError(f"attend_device: q dtype {q.dtype} != cache dtype {self.dtype}")
        if q.stride(-1) != 1:
            q = q.contiguous()
        n_q = q.shape[1]
        out = torch.empty((1, n_q, 1, self.head_dim), dtype=self.dtype, device=self.device)
        scale = self.head_dim ** -0.5 if scale is None else scale
        lib = _lib.load()
        cap = self._dev_capacity
        split = lib.snapmind_paged_gqa_decode_split_tokens(1, self.n_heads, cap, self.block_size)
        need = lib.snapmind_paged_gqa_decode_workspace_bytes(1, n_q, self.n_heads, self.head_dim, cap, split)
        ws = self._workspace.get(1, self.n_heads, need)
        status = lib.snapmind_paged_gqa_decode(
            q.data_ptr(), q.stride(2), q.stride(1),
            self._k_buffer.data_ptr(), self._v_buffer.data_ptr(), _lib.dtype_code(self.dtype),
            self._tables_dev[layer_idx].data_ptr(), 0, self.max_blocks, self._dev_len_p1.data_ptr(),
            out.data_ptr(), out.stride(2), out.stride(1),
            float(scale), 1, n_q, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
            cap, split, 0, ws.data_ptr(), ws.numel(), self._err.data_ptr(),
            self._stream(),
        )  # fmt: skip
        _lib.check(status, "PagedKVCache.attend_device")
        return out

    def advance_device_step(self) -> None:
        """Move the device counters to the next token (two device adds)."""
        self._dev_len.add_(1)
        self._dev_len_p1.add_(1)

    def end_device_steps(self, n_done: int) -> None:
        """Account the ``n_done`` device steps on the host; must equal the steps begun."""
        if self._dev_len is None:
            raise RuntimeError("PagedKVCache: no device steps active")
        if n_done != self._dev_steps:
            raise ValueError(f"PagedKVCache.end_device_steps: {n_done} steps run, {self._dev_steps} begun")
        for layer_idx in range(self.n_layers):
            self._slot_counts[layer_idx] += n_done
        self._dev_len = self._dev_len_p1 = None
        self._dev_steps = self._dev_capacity = 0
        self._version += 1

    # ------------------------------------------------------- introspection
    def block_tables(self) -> list[list[int]]:
        """Copy of the per-layer block tables (host lists)."""
        return [list(bt) for bt in self._block_tables]


class PagedLayerView(MutableMapping):
    """The ``kv_cache`` dict of one layer, backed by a :class:`PagedKVCache`.

    Reads follow the reference's ``layer_dicts`` entries: keys ``"k"`` and
    ``"v"`` always present, ``None`` while the layer is empty, else the layer's
    ``(1, H, T, D)`` contents (one gather for both, reused until the cache
    changes).  Writes follow the protocol of the reference attention layers
    (snapmind/layers/attention/gqa.py:62-67): ``kv_cache["k"], kv_cache["v"] =
    cat(cached, new)``; the rows past the cached length are stored (appended
    on the GPU) once both tensors are assigned.  Attention plugins of this
    package recognise the view and append and attend without a gather.
    """

    KEYS = ("k", "v")

    def __init__(self, cache: PagedKVCache, layer_idx: int):
        self.cache, self.layer_idx = cache, layer_idx
        self._snap: tuple[int, torch.Tensor, torch.Tensor] | None = None
        self._pending: torch.Tensor | None = None

    def __getitem__(self, key):
        if key not in self.KEYS:
            raise KeyError(key)
        if self.cache.num_tokens(self.layer_idx) == 0:
            return None
        if self._snap is None or self._snap[0] != self.cache._version:
            k, v = self.cache.fetch(self.layer_idx)
            self._snap = (self.cache._version, k, v)
        return self._snap[1] if key == "k" else self._snap[2]

    def __setitem__(self, key, value):
        if key == "k":
            self._pending = value
            return
        if key != "v" or self._pending is None:
            raise KeyError(f"PagedLayerView expects 'k' then 'v' assignments, got {key!r}")
        k, v = self._pending, value
        self._pending = None
        n = self.cache.num_tokens(self.layer_idx)
        total = k.shape[-2]
        if k.shape[0] != 1 or v.shape[-2] != total:
            raise ValueError("PagedLayerView: expected (1, H, T, D) key and value of one length")
        if total < n:
            raise ValueError(f"PagedLayerView: the cache holds {n} tokens, got {total}; it cannot shrink")
        if total > n:
            self.cache.store(self.layer_idx, k[:, :, n:], v[:, :, n:], n)

    def __delitem__(self, key):
        raise TypeError("PagedLayerView entries cannot be deleted")

    def __iter__(self):
        return iter(self.KEYS)

    def __len__(self):
        return len(self.KEYS)
