"""The KV-cache plugin contract (snapmind/kv_cache/base.py:9-43).

When the reference package is importable, ``KVCacheABC`` here IS the
reference's class, so every cache of this package is a real subclass of it and
``isinstance(cache, snapmind.kv_cache.base.KVCacheABC)`` holds.  Without the
reference (a serving host that ships only this package) a stand-in with the
same six abstract methods takes its place:
``store(layer_idx, key, value, seq_pos)``, ``fetch(layer_idx) -> (k, v)``,
``evict(tokens_to_keep)``, ``reset()``, ``memory_usage() -> dict`` and
``layer_dicts() -> {layer: {"k": ..., "v": ...}}``.
"""
from __future__ import annotations

import abc
from typing import Any

try:
    from snapmind.kv_cache.base import KVCacheABC
    FROM_REFERENCE = True
except ImportError:
    FROM_REFERENCE = False

    class KVCacheABC(abc.ABC):  # type: ignore[no-redef]
        """Stand-in for the reference's KV-cache contract (same abstract methods)."""

        @abc.abstractmethod
        def store(self, layer_idx: int, key, value, seq_pos: int) -> None: ...

        @abc.abstractmethod
        def fetch(self, layer_idx: int): ...

        @abc.abstractmethod
        def evict(self, tokens_to_keep: int) -> None: ...

        @abc.abstractmethod
        def reset(self) -> None: ...

        @abc.abstractmethod
        def memory_usage(self) -> dict: ...

        @abc.abstractmethod
        def layer_dicts(self) -> dict[int, dict[str, Any]]: ...


__all__ = ["KVCacheABC", "FROM_REFERENCE"]
