from .block_manager import BlockManager, BlockTable
from .kv_cache import FP8KVCachePool, KVCachePool, KVCacheShape

__all__ = ["BlockManager", "BlockTable", "FP8KVCachePool", "KVCachePool", "KVCacheShape"]
