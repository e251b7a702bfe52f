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
        self.device = self.key.device  # "cuda" resolved to its index, as input tensors report it

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


class FP8KVCachePool:
    """FP8 paged KV pool: the layout of :class:`KVCachePool` with one byte per element.

    ``key``/``value`` are uint8 ``[layers, num_blocks, block_size, kv_heads,
    head_dim]`` tensors of OCP FP8 codes (``kv_format`` "e4m3" or "e5m2") with one
    fp32 scale for keys and one for values: an element ``x`` is stored as
    ``fp8(x * (1/scale))`` and read as ``code * scale``.  It holds twice the tokens
    of a bf16 pool in the same memory.  The reference has no FP8 pool; the method
    names follow :class:`KVCachePool` (kv_cache.py:25-166) where they have a
    counterpart there, and :meth:`attend` runs the decode attention of one layer.
    """

    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_dim, *, k_scale, v_scale,
                 kv_format="e4m3", device="cuda"):
        from ..kernels.fp8 import FORMATS, _scale

        values = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        if any(value <= 0 for value in values):
            raise ValueError("all KV cache dimensions must be positive")
        if kv_format not in FORMATS:
            raise ValueError("kv_format must be 'e4m3' or 'e5m2'")
        if head_dim % 2:
            raise ValueError("an fp8 pool needs an even head_dim (copy-on-write moves 16-bit words)")
        self.shape = KVCacheShape(*values)
        self.kv_format = kv_format
        self.k_scale, self.v_scale = _scale(k_scale, "k_scale"), _scale(v_scale, "v_scale")
        self.device = torch.device(device)
        self.key = torch.zeros(values, dtype=torch.uint8, device=self.device)
        self.value = torch.zeros_like(self.key)
        self.device = self.key.device  # "cuda" resolved to its index, as input tensors report it

    @property
    def memory_bytes(self) -> int:
        return self.key.numel() * 2

    def _block_ids(self, block_ids):
        ids = torch.as_tensor(block_ids, dtype=torch.long, device=self.device).flatten()
        if ids.numel() and bool(((ids < 0) | (ids >= self.shape.num_blocks)).any()):
            raise IndexError("physical block id out of range")
        return ids

    def _layer(self, layer):
        if layer < 0 or layer >= self.shape.num_layers:
            raise IndexError("layer out of range")

    def write_slots(self, layer, slot_mapping, key, value, *, validate=True) -> None:
        """Quantise ``key``/``value`` ``[tokens, kv_heads, head_dim]`` into rows ``slot_mapping`` of a layer."""
        from ..kernels.fp8 import write_kv_cache_slots_fp8

        self._layer(layer)
        write_kv_cache_slots_fp8(self.key[layer], self.value[layer], slot_mapping, key, value, self.k_scale,
                                 self.v_scale, kv_format=self.kv_format, validate=validate)

    def write_cuda(self, layer, block_ids, token_offset, key, value, *, validate=True) -> None:
        """Quantise a contiguous token range across pages (the range write of kv_cache.py:123-145)."""
        if key.shape != value.shape or key.ndim != 3:
            raise ValueError("key and value must both have shape [tokens, kv_heads, head_dim]")
        self._layer(layer)
        ids = self._block_ids(block_ids)
        if token_offset < 0 or token_offset + key.shape[0] > ids.numel() * self.shape.block_size:
            raise ValueError("write exceeds supplied block table capacity")
        if key.device != self.device or value.device != self.device:
            raise ValueError("CUDA KV write inputs must be on the cache device")
        bs = self.shape.block_size
        positions = torch.arange(key.shape[0], device=self.device, dtype=torch.long) + int(token_offset)
        slots = ids[positions // bs] * bs + positions % bs
        self.write_slots(layer, slots, key, value, validate=False)

    write = write_cuda

    def attend(self, layer, query, block_tables, context_lens, *, validate=True, workspace=None):
        """Decode attention of one layer over this pool (``paged_attention_fp8``)."""
        from ..kernels.fp8 import paged_attention_fp8

        self._layer(layer)
        return paged_attention_fp8(query, self.key[layer], self.value[layer], block_tables, context_lens,
                                   self.shape.block_size, self.k_scale, self.v_scale, kv_format=self.kv_format,
                                   validate=validate, workspace=workspace)

    def gather(self, layer, block_ids, token_count, dtype=torch.float32):
        """Dequantised logical prefix of a block table as ``[tokens, kv_heads, head_dim]``."""
        if token_count < 0:
            raise ValueError("token_count cannot be negative")
        self._layer(layer)
        ids = self._block_ids(block_ids)
        if token_count > ids.numel() * self.shape.block_size:
            raise ValueError("token_count exceeds supplied block table capacity")
        view = torch.float8_e4m3fn if self.kv_format == "e4m3" else torch.float8_e5m2
        rows = (-1, self.shape.num_kv_heads, self.shape.head_dim)
        key = self.key[layer, ids].reshape(rows)[:token_count].view(view).to(dtype) * self.k_scale
        value = self.value[layer, ids].reshape(rows)[:token_count].view(view).to(dtype) * self.v_scale
        return key, value

    def copy_blocks(self, pairs) -> None:
        """Apply copy-on-write ``(src, dst)`` pairs to every layer of both pools (byte moves)."""
        copy_blocks(self.key.view(torch.bfloat16), self.value.view(torch.bfloat16), pairs)
