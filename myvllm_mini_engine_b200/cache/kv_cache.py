"""Paged KV pool storage (layout of ``mini_engine/cache/kv_cache.py:25-166``).

``key``/``value`` are contiguous ``[layers, num_blocks, block_size, kv_heads,
head_dim]`` tensors; the operators receive the per-layer views ``key[layer]``.
Writes go through the libminikv scatter kernel; ``copy_blocks`` applies the
copy-on-write pairs produced by ``BlockManager.prepare_write``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..kernels.data import copy_blocks, write_kv_cache


@dataclass(frozen=True)
class KVCacheShape:
    num_layers: int
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_dim: int


class KVCachePool:
    """Preallocated key/value tensors indexed by physical block id (kv_cache.py:25-52)."""

    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_dim, *,
                 dtype=torch.bfloat16, device="cuda"):
        values = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        if any(value <= 0 for value in values):
            raise ValueError("all KV cache dimensions must be positive")
        self.shape = KVCacheShape(*values)
        self.dtype = dtype
        self.device = torch.device(device)
        self.key = torch.empty(values, dtype=dtype, device=self.device)
        self.value = torch.empty_like(self.key)

    @property
    def numel(self) -> int:
        return self.key.numel() * 2

    @property
    def memory_bytes(self) -> int:
        return self.numel * self.key.element_size()

    def _block_ids(self, block_ids):
        ids = torch.as_tensor(block_ids, dtype=torch.long, device=self.device).flatten()
        if ids.numel() and bool(((ids < 0) | (ids >= self.shape.num_blocks)).any()):
            raise IndexError("physical block id out of range")
        return ids

    def clear(self, block_ids=None) -> None:
        """Zero all blocks or only the listed ones (kv_cache.py:68-80)."""
        if block_ids is None:
            self.key.zero_()
            self.value.zero_()
            return
        if not block_ids:
            return
        ids = self._block_ids(block_ids)
        self.key.index_fill_(1, ids, 0)
        self.value.index_fill_(1, ids, 0)

    def write_cuda(self, layer, block_ids, token_offset, key, value, *, validate=True) -> None:
        """Write a contiguous token range across pages (kv_cache.py:123-145)."""
        if key.shape != value.shape or key.ndim != 3:
            raise ValueError("key and value must both have shape [tokens, kv_heads, head_dim]")
        if layer < 0 or layer >= self.shape.num_layers:
            raise IndexError("layer out of range")
        ids = self._block_ids(block_ids)
        if token_offset < 0 or token_offset + key.shape[0] > ids.numel() * self.shape.block_size:
            raise ValueError("write exceeds supplied block table capacity")
        if key.device != self.device or value.device != self.device or key.dtype != self.dtype or value.dtype != self.dtype:
            raise ValueError("CUDA KV write inputs must match cache device and dtype")
        write_kv_cache(self.key[layer], self.value[layer], ids, token_offset, key, value,
                       self.shape.block_size, backend="cuda", validate=validate)

    write = write_cuda

    def gather(self, layer, block_ids, token_count):
        """Logical prefix of a block table as ``[tokens, kv_heads, head_dim]`` (kv_cache.py:147-166)."""
        if token_count < 0:
            raise ValueError("token_count cannot be negative")
        if layer < 0 or layer >= self.shape.num_layers:
            raise IndexError("layer out of range")
        ids = self._block_ids(block_ids)
        if token_count > ids.numel() * self.shape.block_size:
            raise ValueError("token_count exceeds supplied block table capacity")
        if token_count == 0:
            empty = (0, self.shape.num_kv_heads, self.shape.head_dim)
            return (torch.empty(empty, dtype=self.dtype, device=self.device),) * 2
        key = self.key[layer, ids].reshape(-1, self.shape.num_kv_heads, self.shape.head_dim)[:token_count]
        value = self.value[layer, ids].reshape(-1, self.shape.num_kv_heads, self.shape.head_dim)[:token_count]
        return key, value

    def copy_blocks(self, pairs) -> None:
        """Apply copy-on-write ``(src, dst)`` pairs to every layer of both pools."""
        copy_blocks(self.key, self.value, pairs)
