"""The KV-cache plugin contract, restated from snapmind/kv_cache/base.py:9-43.

``store(layer_idx, key, value, seq_pos)``, ``fetch(layer_idx) -> (k, v)``,
``evict(tokens_to_keep)``, ``reset()``, ``memory_usage() -> dict`` and
``layer_dicts() -> {layer: {"k": ..., "v": ...}}`` — same names, argument
meaning and return shapes, so the B200 plugins swap in by registry key.
"""
from __future__ import annotations

import abc
from typing import Any

import torch


class KVCacheABC(abc.ABC):
    """Base class for KV cache strategies."""

    @abc.abstractmethod
    def store(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, seq_pos: int) -> None:
        """Store *key* and *value* tensors for the given layer at *seq_pos*."""

    @abc.abstractmethod
    def fetch(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Return ``(keys, values)`` for the given layer, concatenated along the sequence dim."""

    @abc.abstractmethod
    def evict(self, tokens_to_keep: int) -> None:
        """Drop all but the *tokens_to_keep* most recent entries."""

    @abc.abstractmethod
    def reset(self) -> None:
        """Clear all cached data."""

    @abc.abstractmethod
    def memory_usage(self) -> dict:
        """Return a dict with memory/block statistics (keys vary by strategy)."""

    @abc.abstractmethod
    def layer_dicts(self) -> dict[int, dict[str, Any]]:
        """Return the per-layer ``{layer_idx: {"k": tensor, "v": tensor}}`` dict."""
