"""TieredPagedKVCache on the B200: hot chunks on the GPU, cold chunks in pinned host memory.

Drop-in for ``snapmind.kv_cache.tiered.TieredPagedKVCache`` (snapmind/kv_cache/tiered.py:7-232),
registered under the same key ``"tiered"``.  The reference policy is kept
decision for decision (so hot sets, chunk contents and memory accounting are
identical): 64-token chunks keyed by ``seq_pos // chunk_size``; one active
chunk shared by all layers (a token in another chunk finalises it for every
layer); at most ``pool_tokens // chunk_size`` hot chunks, chunk 0 and the
chunks inside the last two chunks' worth of tokens pinned, the highest
unpinned chunk id evicted first; ``score_and_repage`` keeps chunk 0, the tail
chunk and every chunk scoring at least the threshold.

Data placement and movement:
* the active chunk of each layer is a device buffer filled by the
  ``snapmind_kv_append`` kernel;
* a finalised chunk entry is a device tensor while hot and a pinned host
  tensor while cold; offload (D2H) and re-fetch (H2D) are ``cudaMemcpyAsync``
  copies on a dedicated copy stream, ordered against the compute stream with
  stream waits;
* the live view (``layer_dicts`` / ``fetch``) is built by the
  ``snapmind_kv_concat`` kernel from the hot entries in chunk order plus the
  active chunk.

Differences a caller can see: the hot tier and the live tensors are on the CUDA
device whatever ``device`` says ("auto", "cuda" and "cuda:N" are accepted);
stored tensors are copied, not aliased.
"""
from __future__ import annotations

import ctypes

import torch

from snapmind_b200 import _lib
from snapmind_b200.kv_cache.base import KVCacheABC
from snapmind_b200.registry import KV_CACHE


class _Segment(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("row_stride", ctypes.c_int64),
                ("n_tokens", ctypes.c_int32), ("pad_", ctypes.c_int32)]


def _resolve_device(device) -> torch.device:
    if device is None or device == "auto":
        if not torch.cuda.is_available():
            raise RuntimeError("snapmind_b200 TieredPagedKVCache needs a CUDA device")
        return torch.device("cuda", torch.cuda.current_device())
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError(f"snapmind_b200 keeps the hot tier on a CUDA device, got device={device!r}")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def concat_tokens(parts: list[tuple[torch.Tensor, torch.Tensor, int]], device) -> tuple[torch.Tensor, torch.Tensor]:
    """Token-dimension concatenation of (k, v, n_tokens) parts shaped (..., cap, D) on the device."""
    k0 = parts[0][0]
    lead, d = tuple(k0.shape[:-2]), k0.shape[-1]
    total = sum(n for _, _, n in parts)
    k_out = torch.empty(lead + (total, d), dtype=k0.dtype, device=device)
    v_out = torch.empty_like(k_out)
    rows = 1
    for x in lead:
        rows *= x
    segs = (_Segment * len(parts))()
    for i, (k, v, n) in enumerate(parts):
        if tuple(k.shape[:-2]) != lead or k.dtype != k0.dtype or not k.is_contiguous() or not v.is_contiguous():
            raise RuntimeError("tiered cache: chunk entries must share leading shape, dtype and layout")
        segs[i].k, segs[i].v = k.data_ptr(), v.data_ptr()
        segs[i].row_stride, segs[i].n_tokens = k.shape[-2], n
    status = _lib.load().snapmind_kv_concat(ctypes.cast(segs, ctypes.c_void_p), len(parts), rows, d, _lib.dtype_code(k0.dtype),
                                            k_out.data_ptr(), v_out.data_ptr(), total,
                                            _lib.stream_handle(device))
    _lib.check(status, "tiered concat")
    return k_out, v_out


class _Active:
    """Device buffer of one layer's active chunk: (B, H, cap, D), n tokens used."""

    def __init__(self, like: torch.Tensor, cap: int, device):
        shape = tuple(like.shape[:-2]) + (cap, like.shape[-1])
        self.k = torch.empty(shape, dtype=like.dtype, device=device)
        self.v = torch.empty_like(self.k)
        self.n = 0

    @property
    def cap(self) -> int:
        return self.k.shape[-2]


@KV_CACHE.register("tiered")
class TieredPagedKVCache(KVCacheABC):
    def __init__(
        self,
        max_seq_len: int,
        n_layers: int,
        n_heads: int,
        head_dim: int,
        pool_tokens: int = 4096,
        chunk_size: int = 64,
        device: str | torch.device | None = "auto",
    ):
        self.max_seq_len = max_seq_len
        self.n_layers = n_layers
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.chunk_size = chunk_size
        self.max_hot_chunks = max(1, pool_tokens // chunk_size)  # tiered.py:24
        self._device = _resolve_device(device)
        _lib.load()
        self._chunks: dict[int, list[dict[str, torch.Tensor | None]]] = {}
        self._hot_set: set[int] = set()
        self._active: list[_Active | None] = [None] * n_layers
        self._active_chunk_id: int = -1
        self._total_tokens: int = 0
        self._live_dicts: dict[int, dict[str, torch.Tensor | None]] | None = None
        self._copy_stream = torch.cuda.Stream(self._device)
        self._tables: dict[int, torch.Tensor] = {}

    # ------------------------------------------------------------------ copies
    def _to_host(self, t: torch.Tensor) -> torch.Tensor:
        """D2H on the copy stream into pinned memory (ordered after queued compute)."""
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        self._copy_stream.wait_stream(torch.cuda.current_stream(self._device))
        with torch.cuda.stream(self._copy_stream):
            h.copy_(t, non_blocking=True)
        t.record_stream(self._copy_stream)
        return h

    def _to_device(self, t: torch.Tensor) -> torch.Tensor:
        """H2D on the copy stream; the compute stream waits before the next use."""
        d = torch.empty(t.shape, dtype=t.dtype, device=self._device)
        # d's memory may still be read by queued compute-stream work that freed it
        self._copy_stream.wait_stream(torch.cuda.current_stream(self._device))
        with torch.cuda.stream(self._copy_stream):
            d.copy_(t, non_blocking=True)
        d.record_stream(self._copy_stream)
        return d

    def _sync_copies(self) -> None:
        torch.cuda.current_stream(self._device).wait_stream(self._copy_stream)

    def _batch_table(self, batch: int) -> torch.Tensor:
        t = self._tables.get(batch)
        if t is None:
            t = torch.arange(batch, dtype=torch.int32, device=self._device)
            self._tables[batch] = t
        return t

    # ------------------------------------------------------------------ store
    def _append_active(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, t0: int, t1: int) -> None:
        n_new = t1 - t0
        act = self._active[layer_idx]
        if act is not None and (tuple(act.k.shape[:-2]) != tuple(key.shape[:-2]) or act.k.dtype != key.dtype):
            raise RuntimeError("tiered cache: inputs of one chunk must share leading shape and dtype")
        if act is None or act.n + n_new > act.cap:
            cap = max(self.chunk_size, 1)
            need = (act.n if act is not None else 0) + n_new
            while cap < need:
                cap *= 2
            grown = _Active(key, cap, self._device)
            if act is not None and act.n > 0:
                k_old, v_old = concat_tokens([(act.k, act.v, act.n)], self._device)
                grown.k[..., : act.n, :].copy_(k_old)
                grown.v[..., : act.n, :].copy_(v_old)
                grown.n = act.n
            act = grown
            self._active[layer_idx] = act
        lead = key.shape[:-2]
        batch = 1
        for x in lead[:-1]:
            batch *= x
        heads = lead[-1] if len(lead) else 1
        k3 = key.reshape(batch, heads, key.shape[-2], key.shape[-1]) if key.dim() != 4 else key
        v3 = value.reshape(k3.shape) if value.dim() != 4 else value
        if v3.stride() != k3.stride():
            k3, v3 = k3.contiguous(), v3.contiguous()
        st = k3.stride()
        status = _lib.load().snapmind_kv_append(
            act.k.data_ptr(), act.v.data_ptr(), _lib.dtype_code(act.k.dtype), 0,
            k3[:, :, t0:].data_ptr(), v3[:, :, t0:].data_ptr(), _lib.dtype_code(k3.dtype),
            0, st[0], st[1], st[2],
            self._batch_table(batch).data_ptr(), 1, 0, 1,
            None, act.n,
            1, batch, n_new, heads, k3.shape[-1], act.cap, batch,
            None, _lib.stream_handle(self._device),
        )  # fmt: skip
        _lib.check(status, "TieredPagedKVCache.store")
        act.n += n_new

    def store(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, seq_pos: int) -> None:
        """snapmind/kv_cache/tiered.py:50-73, one append per run of same-chunk tokens."""
        n_tokens = key.shape[-2]
        if key.device != self._device:
            key = key.to(self._device)
        if value.device != self._device:
            value = value.to(self._device)
        if key.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            key, value = key.float(), value.float()
        offset = 0
        while offset < n_tokens:
            cid = (seq_pos + offset) // self.chunk_size
            if cid != self._active_chunk_id:
                self._finalize_active_chunk()
                self._active_chunk_id = cid
                self._active = [None] * self.n_layers
            # tokens offset.. that fall in chunk cid
            end = min(n_tokens, (cid + 1) * self.chunk_size - seq_pos)
            if end <= offset:  # negative positions: one token per chunk id step
                end = offset + 1
            self._append_active(layer_idx, key, value, offset, end)
            offset = end
        self._total_tokens = max(self._total_tokens, seq_pos + n_tokens)

    def _finalize_active_chunk(self) -> None:  # tiered.py:75-93
        if self._active_chunk_id < 0:
            return
        cid = self._active_chunk_id
        entries: list[dict[str, torch.Tensor | None]] = []
        all_empty = True
        for i in range(self.n_layers):
            act = self._active[i]
            if act is not None and act.n > 0:
                all_empty = False
                k, v = concat_tokens([(act.k, act.v, act.n)], self._device)
                entries.append({"k": k, "v": v})
            else:
                entries.append({"k": None, "v": None})
        if not all_empty:
            self._chunks[cid] = entries
            self._hot_set.add(cid)
            self._enforce_pool_limit()

    def _enforce_pool_limit(self) -> None:  # tiered.py:95-106
        if len(self._hot_set) <= self.max_hot_chunks:
            return
        tail_start = max(0, self._total_tokens - 2 * self.chunk_size)
        pinned = {0}
        pinned.update(cid for cid in self._hot_set if cid * self.chunk_size >= tail_start)
        evictable = sorted(self._hot_set - pinned, key=lambda c: -c)
        while len(self._hot_set) > self.max_hot_chunks and evictable:
            cid = evictable.pop(0)
            self._hot_set.discard(cid)
            self._offload_chunk(cid)

    def _offload_chunk(self, cid: int) -> None:  # tiered.py:108-118
        if cid not in self._chunks:
            return
        for entry in self._chunks[cid]:
            if entry["k"] is not None and entry["k"].is_cuda:
                entry["k"] = self._to_host(entry["k"])
                if entry["v"] is not None:
                    entry["v"] = self._to_host(entry["v"])

    def score_and_repage(self, scores: dict, threshold: float = 0.5) -> None:  # tiered.py:120-154
        tail_start = max(0, self._total_tokens - self.chunk_size)
        desired_hot = {0}
        desired_hot.update(cid for cid in self._chunks if cid * self.chunk_size >= tail_start)
        for cid, score in scores.items():
            score_val = score.item() if isinstance(score, torch.Tensor) else score
            if cid in self._chunks and score_val >= threshold:
                desired_hot.add(cid)
        for cid in list(self._hot_set):
            if cid not in desired_hot:
                self._hot_set.discard(cid)
                self._offload_chunk(cid)
        fetched = False
        for cid in desired_hot:
            if cid not in self._hot_set and cid in self._chunks:
                self._hot_set.add(cid)
                for entry in self._chunks[cid]:
                    if entry["k"] is not None and not entry["k"].is_cuda:
                        entry["k"] = self._to_device(entry["k"])
                        if entry["v"] is not None:
                            entry["v"] = self._to_device(entry["v"])
                        fetched = True
        if fetched:
            self._sync_copies()
        self._enforce_pool_limit()
        self._rebuild_live_dicts()

    def _rebuild_live_dicts(self) -> None:  # tiered.py:156-182
        if self._live_dicts is None:
            return
        hot_ids = sorted(self._hot_set)
        for i in range(self.n_layers):
            parts = []
            for cid in hot_ids:
                entry = self._chunks[cid][i]
                if entry["k"] is not None and entry["v"] is not None:
                    parts.append((entry["k"], entry["v"], entry["k"].shape[-2]))
            act = self._active[i]
            if act is not None and act.n > 0:
                parts.append((act.k, act.v, act.n))
            if parts:
                k, v = concat_tokens(parts, self._device)
                self._live_dicts[i]["k"] = k
                self._live_dicts[i]["v"] = v
            else:
                self._live_dicts[i] = {"k": None, "v": None}

    def fetch(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:  # tiered.py:184-191
        if self._live_dicts is not None and layer_idx in self._live_dicts:
            d = self._live_dicts[layer_idx]
            k, v = d.get("k"), d.get("v")
            if k is not None and v is not None:
                return k, v
        return torch.empty(0, device=self._device), torch.empty(0, device=self._device)

    def layer_dicts(self) -> dict[int, dict[str, torch.Tensor | None]]:  # tiered.py:193-199
        result: dict[int, dict[str, torch.Tensor | None]] = {i: {"k": None, "v": None} for i in range(self.n_layers)}
        self._live_dicts = result
        self._rebuild_live_dicts()
        return result

    def evict(self, tokens_to_keep: int) -> None:  # tiered.py:201-202
        pass

    def reset(self) -> None:  # tiered.py:204-211
        self._copy_stream.synchronize()
        self._chunks.clear()
        self._hot_set.clear()
        self._active = [None] * self.n_layers
        self._active_chunk_id = -1
        self._total_tokens = 0
        self._live_dicts = None

    def memory_usage(self) -> dict:  # tiered.py:213-232
        gpu_bytes = 0
        cpu_bytes = 0
        for layers in self._chunks.values():
            for entry in layers:
                k = entry.get("k")
                if k is not None:
                    nbytes = k.numel() * k.element_size()
                    if k.is_cuda:
                        gpu_bytes += nbytes * 2
                    else:
                        cpu_bytes += nbytes * 2
        return {
            "gpu_bytes": gpu_bytes,
            "cpu_bytes": cpu_bytes,
            "hot_chunks": len(self._hot_set),
            "cold_chunks": len(self._chunks) - len(self._hot_set),
            "total_tokens": self._total_tokens,
            "pool_slots": self.max_hot_chunks,
        }

    # ------------------------------------------------------- introspection
    def chunk_layout(self) -> dict[int, list[int | None]]:
        """Per chunk id, the token count of each layer's entry (None when empty)."""
        return {cid: [None if e["k"] is None else int(e["k"].shape[-2]) for e in layers]
                for cid, layers in self._chunks.items()}
