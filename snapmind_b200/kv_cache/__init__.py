"""B200 KV-cache plugins; importing this package registers them in ``KV_CACHE``."""
from snapmind_b200.kv_cache.base import KVCacheABC
from snapmind_b200.kv_cache.paged import PagedKVCache
from snapmind_b200.kv_cache.sliding_window import SlidingWindowKVCache
from snapmind_b200.kv_cache.tiered import TieredPagedKVCache

__all__ = ["KVCacheABC", "PagedKVCache", "SlidingWindowKVCache", "TieredPagedKVCache"]
