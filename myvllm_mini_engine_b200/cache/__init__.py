from .block_manager import BlockManager, BlockTable
from .kv_cache import KVCachePool, KVCacheShape

__all__ = ["BlockManager", "BlockTable", "KVCachePool", "KVCacheShape"]
