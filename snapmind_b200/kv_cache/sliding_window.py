"""SlidingWindowKVCache on the B200: each layer's window as a row of pool blocks.

Drop-in for ``snapmind.kv_cache.sliding_window.SlidingWindowKVCache``
(snapmind/kv_cache/sliding_window.py:9-86), registered under the same key
``"sliding_window"``: the same constructor, ``store`` keeping the newest
``window_size`` tokens of each layer, ``fetch`` returning them as
``(1, H, T, D)`` (two empty tensors for an empty layer), ``evict`` keeping the
newest ``tokens_to_keep`` (``0`` keeps everything, as the reference's
``[..., -0:, :]`` slice does), ``reset``, ``memory_usage`` with the same keys,
and ``layer_dicts``.

Layout (the "ring of blocks" form of the paged pool): K/V live in a pool
``[block][head][slot][dim]`` shared by the layers; layer l holds a table row
of blocks and a start offset ``skip < block_size`` into its first block — the
window is tokens ``[skip, skip + n)`` of the row.  Appending writes rows with
the paged append kernel; trimming the front returns whole blocks to the free
list and advances ``skip``; no K/V byte is moved.  Decode attention reads the
window straight from the pool (``snapmind_paged_gqa_decode_window``: tokens
before ``skip`` masked).

``layer_dicts`` returns views for the model protocol (the reference returns its
internal dicts, which the models grow with ``torch.cat`` in
snapmind/layers/attention/gqa.py:62-67 and trim in
snapmind/models/mistral.py:58-60): reading gives the window; assigning a longer
tensor appends the new rows and keeps the window; assigning a shorter one drops
tokens from the front.  The ``gqa_paged`` attention plugin appends and attends
through them without a gather.

Differences a caller can see: one sequence (``key[0]``), like the paged cache;
tensors live on the CUDA device; ``store`` keeps ``value`` rows as V — the
reference concatenates the cached keys with the new values there
(sliding_window.py:27), a defect that the models' own path (dict growth) does
not reach.
"""
from __future__ import annotations

from collections.abc import MutableMapping

import torch

from snapmind_b200 import _lib
from snapmind_b200.kv_cache.base import KVCacheABC
from snapmind_b200.kv_cache.paged import _default_device
from snapmind_b200.registry import KV_CACHE

_KERNEL_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


@KV_CACHE.register("sliding_window")
class SlidingWindowKVCache(KVCacheABC):
    def __init__(self, max_seq_len: int, n_layers: int, n_heads: int, head_dim: int, window_size: int = 4096, *,
                 block_size: int = 16, dtype: torch.dtype | None = None, device: torch.device | str | None = None):
        if window_size <= 0:
            raise ValueError("window_size must be positive")
        self.max_seq_len = max_seq_len
        self.n_layers, self.n_heads, self.head_dim = n_layers, n_heads, head_dim
        self.window_size = window_size
        self.block_size = block_size
        self.device = torch.device(device) if device is not None else _default_device()
        _lib.require_cuda(self.device)
        _lib.load()
        self.dtype = dtype  # fixed by the first store when None
        # a row holds up to two windows (a window plus up to window_size new tokens
        # before the trim) and a partly used first and last block
        self.row_blocks = (2 * window_size + block_size - 1) // block_size + 2
        self.max_blocks = n_layers * self.row_blocks
        self._k: torch.Tensor | None = None
        self._v: torch.Tensor | None = None
        self._tables_dev = torch.zeros((n_layers, self.row_blocks), dtype=torch.int32, device=self.device)
        self._lens_dev = torch.zeros(n_layers, dtype=torch.int32, device=self.device)   # skip + n
        self._starts_dev = torch.zeros(n_layers, dtype=torch.int32, device=self.device)  # skip
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._workspace = _lib.DecodeWorkspace(self.device)
        self._version = 0
        self._reset_host()

    # ------------------------------------------------------------------ state
    def _reset_host(self) -> None:
        self._free = list(range(self.max_blocks - 1, -1, -1))
        self._tables: list[list[int]] = [[] for _ in range(self.n_layers)]
        self._skip = [0] * self.n_layers
        self._n = [0] * self.n_layers

    def _ensure_pool(self, dtype: torch.dtype) -> None:
        if self._k is not None:
            return
        if self.dtype is None:
            self.dtype = dtype if dtype in _KERNEL_DTYPES else torch.float32
        shape = (self.max_blocks, self.n_heads, self.block_size, self.head_dim)
        self._k = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self._v = torch.zeros(shape, dtype=self.dtype, device=self.device)

    def _sync_layer(self, layer: int) -> None:
        row = self._tables[layer]
        if row:
            self._tables_dev[layer, : len(row)].copy_(torch.tensor(row, dtype=torch.int32))
        vals = torch.tensor([self._skip[layer] + self._n[layer], self._skip[layer]], dtype=torch.int32)
        self._lens_dev[layer].copy_(vals[0])
        self._starts_dev[layer].copy_(vals[1])

    def num_tokens(self, layer: int) -> int:
        return self._n[layer]

    def check_device_errors(self) -> None:
        word = int(self._err.item())
        if word:
            self._err.zero_()
            _lib.raise_device_error(word, "SlidingWindowKVCache")

    # ---------------------------------------------------------- primitives
    def _append(self, layer: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append rows ``key[0, :, t, :]`` after the window (no trim)."""
        n_new = key.shape[-2]
        if n_new == 0:
            return
        if key.shape[1] != self.n_heads or key.shape[-1] != self.head_dim:
            raise ValueError(f"SlidingWindowKVCache: expected (1, {self.n_heads}, T, {self.head_dim}), "
                             f"got {tuple(key.shape)}")
        self._ensure_pool(key.dtype)
        bs, row = self.block_size, self._tables[layer]
        end = self._skip[layer] + self._n[layer] + n_new
        need = (end + bs - 1) // bs
        if need > self.row_blocks:
            raise ValueError(f"SlidingWindowKVCache: {self._n[layer]} + {n_new} tokens exceed a row of "
                             f"{self.row_blocks} blocks; append at most window_size tokens to a window")
        while len(row) < need:
            if not self._free:
                raise RuntimeError(_lib.OUT_OF_BLOCKS_MSG)
            row.append(self._free.pop())
        slot0 = self._skip[layer] + self._n[layer]
        self._n[layer] += n_new
        self._sync_layer(layer)
        k = key[0].to(self.device)
        v = value[0].to(self.device)
        if k.dtype not in _KERNEL_DTYPES:
            k, v = k.to(self.dtype), v.to(self.dtype)
        if k.stride(-1) != 1 or v.stride() != k.stride() or v.dtype != k.dtype:
            k, v = k.contiguous(), v.to(k.dtype).contiguous()
        status = _lib.load().snapmind_kv_append(
            self._k.data_ptr(), self._v.data_ptr(), _lib.dtype_code(self.dtype), 0,
            k.data_ptr(), v.data_ptr(), _lib.dtype_code(k.dtype),
            0, 0, k.stride(0), k.stride(1),
            self._tables_dev[layer].data_ptr(), 0, 0, self.row_blocks,
            None, slot0,
            1, 1, n_new, self.n_heads, self.head_dim, bs, self.max_blocks,
            self._err.data_ptr(), _lib.stream_handle(self.device),
        )  # fmt: skip
        _lib.check(status, "SlidingWindowKVCache.store")
        self._version += 1

    def _trim(self, layer: int, keep: int) -> None:
        """Keep the newest ``keep`` tokens: whole front blocks go back to the free list."""
        n = self._n[layer]
        if keep >= n:
            return
        bs = self.block_size
        start = self._skip[layer] + (n - keep)
        drop = start // bs
        row = self._tables[layer]
        for blk in row[:drop]:
            self._free.append(blk)
        del row[:drop]
        self._skip[layer] = start - drop * bs
        self._n[layer] = keep
        if keep == 0:
            self._free.extend(row)
            row.clear()
            self._skip[layer] = 0
        self._sync_layer(layer)
        self._version += 1

    # --------------------------------------------------------------------- API
    def store(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, seq_pos: int) -> None:
        """Append ``key``/``value`` rows (``(1, H, T, D)``) and keep the newest
        ``window_size`` tokens (snapmind/kv_cache/sliding_window.py:19-38)."""
        w = self.window_size
        if key.shape[-2] >= w:  # only the newest window of the new rows survives
            self._trim(layer_idx, 0)
            key, value = key[:, :, -w:], value[:, :, -w:]
        self._append(layer_idx, key, value)
        self._trim(layer_idx, w)

    def fetch(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        n = self._n[layer_idx]
        if n == 0:
            # the reference returns two empty float32 tensors (sliding_window.py:44-48)
            return (torch.empty(0, dtype=torch.float32, device=self.device),
                    torch.empty(0, dtype=torch.float32, device=self.device))
        skip = self._skip[layer_idx]
        total = skip + n
        k = torch.empty((1, self.n_heads, total, self.head_dim), dtype=self.dtype, device=self.device)
        v = torch.empty_like(k)
        status = _lib.load().snapmind_kv_gather(
            self._k.data_ptr(), self._v.data_ptr(), _lib.dtype_code(self.dtype), 0,
            k.data_ptr(), v.data_ptr(), 0, k.numel(),
            self._tables_dev[layer_idx].data_ptr(), 0, 0, self.row_blocks,
            None, total,
            1, 1, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
            self._err.data_ptr(), _lib.stream_handle(self.device),
        )  # fmt: skip
        _lib.check(status, "SlidingWindowKVCache.fetch")
        if skip:
            k, v = k[:, :, skip:].contiguous(), v[:, :, skip:].contiguous()
        return k, v

    def evict(self, tokens_to_keep: int) -> None:
        """Keep the newest ``tokens_to_keep`` tokens per layer; like the reference's
        ``[..., -tokens_to_keep:, :]`` slice, 0 keeps every token."""
        if tokens_to_keep <= 0:
            return
        for layer in range(self.n_layers):
            self._trim(layer, tokens_to_keep)

    def reset(self) -> None:
        self._reset_host()
        self._tables_dev.zero_()
        self._lens_dev.zero_()
        self._starts_dev.zero_()
        self._version += 1

    def memory_usage(self) -> dict:
        """``num_tokens`` and ``total_bytes`` of the held K and V windows
        (sliding_window.py:65-78 counts its tensors' bytes)."""
        n = sum(self._n)
        elem = self._k.element_size() if self._k is not None else 4
        return {"num_tokens": n, "total_bytes": 2 * n * self.n_heads * self.head_dim * elem}

    def layer_dicts(self) -> dict[int, "SlidingLayerView"]:
        return {i: SlidingLayerView(self, i) for i in range(self.n_layers)}

    # ------------------------------------------------------------- attention
    def attend(self, layer_idx: int, q: torch.Tensor, lens: torch.Tensor, starts: torch.Tensor,
               scale: float | None = None) -> torch.Tensor:
        """Attention of queries ``q`` ``(1, Hq, T, D)`` over the layer's row: query t
        attends to rows ``[starts[t], lens[t])`` (int32 device tensors of T entries,
        positions in the layer's table row, whose first ``skip`` rows precede the
        window)."""
        if q.dtype != self.dtype:
            raise TypeError(f"attend: q dtype {q.dtype} != cache dtype {self.dtype}")
        n_q, n_t = q.shape[1], q.shape[2]
        out = torch.empty((1, n_q, n_t, self.head_dim), dtype=self.dtype, device=self.device)
        if n_t == 0:
            return out
        if q.stride(-1) != 1:
            q = q.contiguous()
        total = self._skip[layer_idx] + self._n[layer_idx]
        scale = self.head_dim ** -0.5 if scale is None else scale
        lib = _lib.load()
        split = lib.snapmind_paged_gqa_decode_split_tokens(n_t, self.n_heads, total, self.block_size)
        need = lib.snapmind_paged_gqa_decode_workspace_bytes(n_t, n_q, self.n_heads, self.head_dim, total, split)
        ws = self._workspace.get(n_t, self.n_heads, need)
        status = lib.snapmind_paged_gqa_decode_window(
            q.data_ptr(), q.stride(2), q.stride(1),
            self._k.data_ptr(), self._v.data_ptr(), _lib.dtype_code(self.dtype),
            self._tables_dev[layer_idx].data_ptr(), 0, self.row_blocks, lens.data_ptr(), starts.data_ptr(),
            out.data_ptr(), out.stride(2), out.stride(1),
            float(scale), n_t, n_q, self.n_heads, self.head_dim, self.block_size, self.max_blocks,
            total, split, 0, ws.data_ptr(), ws.numel(), self._err.data_ptr(),
            _lib.stream_handle(self.device),
        )  # fmt: skip
        _lib.check(status, "SlidingWindowKVCache.attend")
        return out

    def block_tables(self) -> list[list[int]]:
        return [list(r) for r in self._tables]


class SlidingLayerView(MutableMapping):
    """The ``kv_cache`` dict of one layer, backed by a :class:`SlidingWindowKVCache`.

    Reads give the window (``None`` while empty).  Assignments follow the
    models' protocol: ``kv_cache["k"], kv_cache["v"] = k, v`` with ``k`` longer
    than the window held appends the new rows (then keeps ``window_size``); a
    shorter ``k`` keeps its length of newest tokens (the trim of
    snapmind/models/mistral.py:58-60)."""

    KEYS = ("k", "v")

    def __init__(self, cache: SlidingWindowKVCache, layer_idx: int):
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
            raise KeyError(f"SlidingLayerView expects 'k' then 'v' assignments, got {key!r}")
        k, v = self._pending, value
        self._pending = None
        n, total = self.cache.num_tokens(self.layer_idx), k.shape[-2]
        if total > n:
            self.cache.store(self.layer_idx, k[:, :, n:], v[:, :, n:], n)
        else:
            self.cache._trim(self.layer_idx, total)

    def __delitem__(self, key):
        raise TypeError("SlidingLayerView entries cannot be deleted")

    def __iter__(self):
        return iter(self.KEYS)

    def __len__(self):
        return len(self.KEYS)
