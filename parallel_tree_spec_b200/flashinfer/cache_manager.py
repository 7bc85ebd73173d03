"""``parallel_tree_spec.flashinfer.cache_manager`` under its reference import path."""
from ..cache_manager import KvCacheBatchPosition, KvCachePool, RequestKvCache, getKvCacheBatchPosition  # noqa: F401
