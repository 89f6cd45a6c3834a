"""Registration of the B200 plugins into snapmind's own registries.

The reference creates its KV caches, attention layers and indexer by string
key from three registries (snapmind/core/registry.py:92-111: ``KV_CACHE``,
``ATTENTION``, ``INDEXER``); its engine, for one, calls
``INDEXER.create("lookahead_sparse", ...)`` (snapmind/engine/generate.py:51).
:func:`register_with_snapmind` puts this package's classes under the keys a
snapmind config names, so an unchanged snapmind program picks them up:

==================  ===================  ====================================
registry            key                  class
==================  ===================  ====================================
``KV_CACHE``        ``"paged"``          ``kv_cache.paged.PagedKVCache``
``KV_CACHE``        ``"tiered"``         ``kv_cache.tiered.TieredPagedKVCache``
``KV_CACHE``        ``"sliding_window"`` ``kv_cache.sliding_window.SlidingWindowKVCache``
``ATTENTION``       ``"gqa_paged"``      ``attention.PagedGroupedQueryAttention``
``INDEXER``         ``"lookahead_sparse"`` ``indexer.LookaheadSparseIndexer``
==================  ===================  ====================================

The reference registers its own classes under the first four of those keys
when their modules are imported, and a second import-time registration of a
taken key raises ``RegistryError``.  So the reference modules are imported
first (their registrations happen once, now), then the B200 classes replace
them with ``override=True``.  A snapmind module imported afterwards is already
loaded and registers nothing again.

Membership in the reference's class hierarchy: when snapmind was importable as
this package was imported, the B200 classes subclass the reference's
``KVCacheABC`` / ``AttentionABC`` / ``IndexerABC`` directly.  If snapmind only
became importable later, this function declares them virtual subclasses
(``ABCMeta.register``), so ``isinstance`` against the reference contracts holds
either way.
"""
from __future__ import annotations

import importlib

_REFERENCE_MODULES = (
    "snapmind.kv_cache.paged",
    "snapmind.kv_cache.tiered",
    "snapmind.kv_cache.sliding_window",
    "snapmind.layers.indexer.lookahead",
)


def plugin_table() -> list[tuple[str, str, type, str]]:
    """(registry name, key, B200 class, reference contract "module:Class") rows."""
    from snapmind_b200.attention import PagedGroupedQueryAttention
    from snapmind_b200.indexer import LookaheadSparseIndexer
    from snapmind_b200.kv_cache import PagedKVCache, SlidingWindowKVCache, TieredPagedKVCache

    kv = "snapmind.kv_cache.base:KVCacheABC"
    return [
        ("KV_CACHE", "paged", PagedKVCache, kv),
        ("KV_CACHE", "tiered", TieredPagedKVCache, kv),
        ("KV_CACHE", "sliding_window", SlidingWindowKVCache, kv),
        ("ATTENTION", "gqa_paged", PagedGroupedQueryAttention, "snapmind.layers.attention.base:AttentionABC"),
        ("INDEXER", "lookahead_sparse", LookaheadSparseIndexer, "snapmind.layers.indexer.base:IndexerABC"),
    ]


def _contract(path: str) -> type:
    module, name = path.split(":")
    return getattr(importlib.import_module(module), name)


def register_with_snapmind(override: bool = True) -> dict[str, list[str]]:
    """Register every B200 plugin into snapmind's registries; returns the keys per registry.

    Raises ``ImportError`` when snapmind is not importable.  With
    ``override=False`` a key the reference already holds raises snapmind's
    ``RegistryError``, as its own ``register`` does.
    """
    registry = importlib.import_module("snapmind.core.registry")
    for name in _REFERENCE_MODULES:
        importlib.import_module(name)
    done: dict[str, list[str]] = {}
    for reg_name, key, cls, contract in plugin_table():
        base = _contract(contract)
        if not issubclass(cls, base):
            base.register(cls)
        getattr(registry, reg_name).register(key, cls, override=override)
        done.setdefault(reg_name, []).append(key)
    return done


__all__ = ["plugin_table", "register_with_snapmind"]
