"""Oracle: the sliding-window KV cache (snapmind/kv_cache/sliding_window.py:9-86) on numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

``v_from_cached_k=True`` reproduces the reference exactly, including its store
building V from the cached keys (sliding_window.py:27) — the form checked
against the reference's own goldens; ``False`` is the same cache storing V,
the form the B200 plugin implements.
"""
from __future__ import annotations

import numpy as np


class SlidingWindowOracle:
    def __init__(self, n_layers, window_size, v_from_cached_k=False):  # :11-17
        self.n_layers = n_layers
        self.window_size = window_size
        self.v_from_cached_k = v_from_cached_k
        self.caches = [{"k": None, "v": None} for _ in range(n_layers)]

    def store(self, layer, key, value):  # :19-29
        c = self.caches[layer]
        if c["k"] is None:
            c["k"], c["v"] = key.copy(), value.copy()
        else:
            c["v"] = np.concatenate([c["k"] if self.v_from_cached_k else c["v"], value], axis=-2)
            c["k"] = np.concatenate([c["k"], key], axis=-2)
        self._trim(layer)

    def _trim(self, layer):  # :31-38
        c = self.caches[layer]
        if c["k"] is not None and c["k"].shape[-2] > self.window_size:
            c["k"] = c["k"][..., -self.window_size:, :]
            c["v"] = c["v"][..., -self.window_size:, :]

    def fetch(self, layer):  # :40-49
        c = self.caches[layer]
        if c["k"] is None:
            return np.empty(0, np.float32), np.empty(0, np.float32)
        return c["k"], c["v"]

    def evict(self, tokens_to_keep):  # :51-58 (a slice [-0:] keeps everything)
        for c in self.caches:
            if c["k"] is not None:
                c["k"] = c["k"][..., -tokens_to_keep:, :]
                c["v"] = c["v"][..., -tokens_to_keep:, :]

    def reset(self):  # :60-62
        self.caches = [{"k": None, "v": None} for _ in range(self.n_layers)]

    def memory_usage(self):  # :64-77
        total, n = 0, 0
        for c in self.caches:
            if c["k"] is not None:
                total += c["k"].nbytes + c["v"].nbytes
                n += c["k"].shape[-2]
        return {"num_tokens": n, "total_bytes": total}
