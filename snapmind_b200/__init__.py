"""snapmind_b200 — the KV-cache hot path of snapmind as hand-written sm_100a kernels.

Importing the package registers the B200 plugins in this package's registries
(``snapmind_b200.registry.KV_CACHE`` …) under the reference's keys.  The CUDA
library is loaded on first use; there is no CPU fallback.
"""
from snapmind_b200 import kv_cache  # noqa: F401  (registers "paged", "tiered", "sliding_window")
from snapmind_b200 import indexer  # noqa: F401  (registers "lookahead_sparse")
from snapmind_b200 import attention  # noqa: F401  (registers "gqa_paged")
from snapmind_b200.attention import PagedGroupedQueryAttention
from snapmind_b200.kv_cache import PagedKVCache, SlidingWindowKVCache, TieredPagedKVCache
from snapmind_b200.mla import MLALatentPool, PagedLatentDict
from snapmind_b200.paged_pool import PagedKVPool
from snapmind_b200.registry import ATTENTION, INDEXER, KV_CACHE, Registry, RegistryError

__all__ = ["KV_CACHE", "ATTENTION", "INDEXER", "Registry", "RegistryError", "PagedKVPool", "MLALatentPool",
           "PagedLatentDict", "PagedGroupedQueryAttention", "PagedKVCache", "SlidingWindowKVCache",
           "TieredPagedKVCache"]
__version__ = "0.1.0"
