from .cow import copy_on_write, prepare_write
from .kv_cache import FP8KVCachePool, PagedKVPool, PoolShape

__all__ = ["FP8KVCachePool", "PagedKVPool", "PoolShape", "copy_on_write", "prepare_write"]
