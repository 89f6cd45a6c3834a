"""Oracle: the tiered KV cache (snapmind/kv_cache/tiered.py:7-232) on numpy arrays.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Same decisions as the reference, with every chunk entry a numpy array and its
placement tracked by a flag (``dev=True`` where the reference would hold the
tensor on its device, False after ``.to("cpu")``), so memory accounting can be
compared with a cache whose hot tier is really on a GPU.
"""
from __future__ import annotations

import numpy as np


class TieredPagedKVCacheOracle:
    def __init__(self, max_seq_len, n_layers, n_heads, head_dim, pool_tokens=4096, chunk_size=64):
        self.n_layers = n_layers
        self.chunk_size = chunk_size
        self.max_hot_chunks = max(1, pool_tokens // chunk_size)  # :24
        self.chunks: dict[int, list[dict]] = {}
        self.hot_set: set[int] = set()
        self.active_k = [None] * n_layers
        self.active_v = [None] * n_layers
        self.active_chunk_id = -1
        self.total_tokens = 0
        self.live_dicts = None

    def store(self, layer_idx, key, value, seq_pos):  # :50-73
        n_tokens = key.shape[-2]
        for offset in range(n_tokens):
            cid = (seq_pos + offset) // self.chunk_size
            if cid != self.active_chunk_id:
                self._finalize_active_chunk()
                self.active_chunk_id = cid
                self.active_k = [None] * self.n_layers
                self.active_v = [None] * self.n_layers
            ks = key[..., offset:offset + 1, :]
            vs = value[..., offset:offset + 1, :]
            if self.active_k[layer_idx] is None or self.active_v[layer_idx] is None:
                self.active_k[layer_idx] = ks.copy()
                self.active_v[layer_idx] = vs.copy()
            else:
                self.active_k[layer_idx] = np.concatenate([self.active_k[layer_idx], ks], axis=-2)
                self.active_v[layer_idx] = np.concatenate([self.active_v[layer_idx], vs], axis=-2)
        self.total_tokens = max(self.total_tokens, seq_pos + n_tokens)

    def _finalize_active_chunk(self):  # :75-93
        if self.active_chunk_id < 0:
            return
        entries, all_empty = [], True
        for i in range(self.n_layers):
            k, v = self.active_k[i], self.active_v[i]
            if k is not None and v is not None:
                all_empty = False
                entries.append({"k": k, "v": v, "dev": True})
            else:
                entries.append({"k": None, "v": None, "dev": True})
        if not all_empty:
            self.chunks[self.active_chunk_id] = entries
            self.hot_set.add(self.active_chunk_id)
            self._enforce_pool_limit()

    def _enforce_pool_limit(self):  # :95-106
        if len(self.hot_set) <= self.max_hot_chunks:
            return
        tail_start = max(0, self.total_tokens - 2 * self.chunk_size)
        pinned = {0} | {cid for cid in self.hot_set if cid * self.chunk_size >= tail_start}
        evictable = sorted(self.hot_set - pinned, key=lambda c: -c)
        while len(self.hot_set) > self.max_hot_chunks and evictable:
            cid = evictable.pop(0)
            self.hot_set.discard(cid)
            self._offload_chunk(cid)

    def _offload_chunk(self, cid):  # :108-118
        if cid not in self.chunks:
            return
        for e in self.chunks[cid]:
            if e["k"] is not None:
                e["dev"] = False

    def score_and_repage(self, scores, threshold=0.5):  # :120-154
        tail_start = max(0, self.total_tokens - self.chunk_size)
        desired = {0} | {cid for cid in self.chunks if cid * self.chunk_size >= tail_start}
        for cid, s in scores.items():
            if cid in self.chunks and float(s) >= threshold:
                desired.add(cid)
        for cid in list(self.hot_set):
            if cid not in desired:
                self.hot_set.discard(cid)
                self._offload_chunk(cid)
        for cid in desired:
            if cid not in self.hot_set and cid in self.chunks:
                self.hot_set.add(cid)
                for e in self.chunks[cid]:
                    if e["k"] is not None:
                        e["dev"] = True
        self._enforce_pool_limit()
        self._rebuild_live_dicts()

    def _rebuild_live_dicts(self):  # :156-182
        if self.live_dicts is None:
            return
        hot_ids = sorted(self.hot_set)
        for i in range(self.n_layers):
            kp, vp = [], []
            for cid in hot_ids:
                e = self.chunks[cid][i]
                if e["k"] is not None and e["v"] is not None:
                    kp.append(e["k"])
                    vp.append(e["v"])
            if self.active_k[i] is not None and self.active_v[i] is not None:
                kp.append(self.active_k[i])
                vp.append(self.active_v[i])
            if kp:
                self.live_dicts[i]["k"] = np.concatenate(kp, axis=-2)
                self.live_dicts[i]["v"] = np.concatenate(vp, axis=-2)
            else:
                self.live_dicts[i] = {"k": None, "v": None}

    def fetch(self, layer_idx):  # :184-191
        if self.live_dicts is not None and layer_idx in self.live_dicts:
            d = self.live_dicts[layer_idx]
            if d.get("k") is not None and d.get("v") is not None:
                return d["k"], d["v"]
        return np.empty(0, np.float32), np.empty(0, np.float32)

    def layer_dicts(self):  # :193-199
        self.live_dicts = {i: {"k": None, "v": None} for i in range(self.n_layers)}
        self._rebuild_live_dicts()
        return self.live_dicts

    def evict(self, tokens_to_keep):  # :201-202, a no-op in the reference
        pass

    def reset(self):  # :204-211
        self.chunks.clear()
        self.hot_set.clear()
        self.active_k = [None] * self.n_layers
        self.active_v = [None] * self.n_layers
        self.active_chunk_id = -1
        self.total_tokens = 0
        self.live_dicts = None

    def memory_usage(self, elem_size=4):  # :213-232, device vs host by placement flag
        gpu = cpu = 0
        for layers in self.chunks.values():
            for e in layers:
                if e["k"] is not None:
                    nbytes = e["k"].size * elem_size * 2
                    if e["dev"]:
                        gpu += nbytes
                    else:
                        cpu += nbytes
        return {"gpu_bytes": gpu, "cpu_bytes": cpu, "hot_chunks": len(self.hot_set),
                "cold_chunks": len(self.chunks) - len(self.hot_set), "total_tokens": self.total_tokens,
                "pool_slots": self.max_hot_chunks}

    def chunk_layout(self):
        return {cid: [None if e["k"] is None else int(e["k"].shape[-2]) for e in layers]
                for cid, layers in self.chunks.items()}
