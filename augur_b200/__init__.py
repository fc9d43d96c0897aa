"""augur_b200 — sm_100a KV-cache data movement for the augur inference engine.

Drop-in modules with augur's cache API (same names, signatures, checks and
error messages):

  augur_b200.kv_cache        <- augur/kv_cache.py
  augur_b200.paged_kv_cache  <- augur/paged_kv_cache.py
  augur_b200.prefix_cache    <- augur/prefix_cache.py

plus batched all-layer entry points in augur_b200.batched and sequence
sharding / peer push in augur_b200.sharding and augur_b200.peer, and the
cache's consumers that read the pool in place in augur_b200.attention
(decode and prefill attention) and augur_b200.decode. Every byte of cache
data the device moves goes through libaugur_kv.so (include/augur_kv.h);
there is no CPU fallback.
"""

from ._lib import KVLibraryError
from ._ops import check_status, read_status
from .config import QwenConfig
from .kv_cache import KVCache, format_bytes, kv_cache_nbytes, new_kv_cache, write_kv
from .paged_kv_cache import (
    BlockAllocator,
    PagedKVCache,
    PagedKVCacheState,
    PagedPrefixCache,
    PagedPrefixCacheMatch,
    SequenceBlockTable,
    new_paged_kv_cache,
    read_paged_kv,
    write_paged_kv,
)
from .prefix_cache import PrefixCache, PrefixCacheEntry, cache_prefix, copy_prefix_into_cache

__all__ = [
    "BlockAllocator",
    "KVCache",
    "KVLibraryError",
    "PagedKVCache",
    "PagedKVCacheState",
    "PagedPrefixCache",
    "PagedPrefixCacheMatch",
    "PrefixCache",
    "PrefixCacheEntry",
    "QwenConfig",
    "SequenceBlockTable",
    "cache_prefix",
    "check_status",
    "copy_prefix_into_cache",
    "format_bytes",
    "kv_cache_nbytes",
    "new_kv_cache",
    "new_paged_kv_cache",
    "read_paged_kv",
    "read_status",
    "write_kv",
    "write_paged_kv",
]
