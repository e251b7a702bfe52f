"""KV page pools for this package's own decode step, benchmarks and tests.

The reference runtime keeps its own pool class (``mini_engine/cache/kv_cache.py``);
through :func:`myvllm_mini_engine_b200.integration.install` it calls the kernels
here with that class's per-layer views.  The pools below hold the same layout,
``[layers, num_blocks, block_size, kv_heads, head_dim]`` per tensor
(kv_cache.py:50-52), and expose ``key``, ``value`` and ``shape`` under the same
names, so :class:`~myvllm_mini_engine_b200.engine.qwen3.Qwen3DecodeStep`
accepts either the reference pool or one of these.

* :class:`PagedKVPool`: 16-bit (or fp32) pages.  Both pools live in one
  allocation ``[2, layers, ...]``, so a step's K and V pages of a layer are one
  address range apart and a single free returns them.
* :class:`FP8KVCachePool`: one OCP FP8 byte per element plus a scale per pool.

Page-id checks are done on the host for Python sequences (no device sync) and
with one reduction for device tensors.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ..kernels.data import copy_blocks, write_kv_cache


@dataclass(frozen=True)
class PoolShape:
    """Geometry of a pool; the field names are the ones the reference pool's ``shape`` carries."""

    num_layers: int
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_dim: int

    @property
    def row_elems(self) -> int:
        return self.num_kv_heads * self.head_dim


def _geometry(values) -> PoolShape:
    if any(int(v) <= 0 for v in values):
        raise ValueError("all KV cache dimensions must be positive")
    return PoolShape(*(int(v) for v in values))


def _page_tensor(block_ids, shape: PoolShape, device) -> torch.Tensor:
    """Page ids as a flat int64 tensor on ``device``; IndexError if one is outside the pool."""
    if isinstance(block_ids, torch.Tensor):
        ids = block_ids.reshape(-1).to(device=device, dtype=torch.long)
        if ids.numel():
            lo, hi = torch.aminmax(ids)
            if int(lo) < 0 or int(hi) >= shape.num_blocks:
                raise IndexError("physical block id out of range")
        return ids
    host = np.asarray(list(block_ids), dtype=np.int64).reshape(-1)
    if host.size and (host.min() < 0 or host.max() >= shape.num_blocks):
        raise IndexError("physical block id out of range")
    return torch.from_numpy(host).to(device)


class _Pool:
    shape: PoolShape
    key: torch.Tensor
    value: torch.Tensor

    def _check_layer(self, layer):
        if not 0 <= layer < self.shape.num_layers:
            raise IndexError("layer out of range")

    def _check_range(self, ids, token_offset, tokens):
        if token_offset < 0 or token_offset + tokens > ids.numel() * self.shape.block_size:
            raise ValueError("write exceeds supplied block table capacity")

    @property
    def memory_bytes(self) -> int:
        return (self.key.numel() + self.value.numel()) * self.key.element_size()

    def layer(self, index):
        """``(key, value)`` views of one layer: ``[num_blocks, block_size, kv_heads, head_dim]``."""
        self._check_layer(index)
        return self.key[index], self.value[index]


class PagedKVPool(_Pool):
    """K and V pages of every layer, one contiguous allocation ``[2, layers, blocks, bs, kv_heads, D]``."""

    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_dim, *,
                 dtype=torch.bfloat16, device="cuda"):
        self.shape = _geometry((num_layers, num_blocks, block_size, num_kv_heads, head_dim))
        self.dtype = dtype
        self.storage = torch.empty((2, *map(int, (num_layers, num_blocks, block_size, num_kv_heads, head_dim))),
                                   dtype=dtype, device=device)
        self.key, self.value = self.storage[0], self.storage[1]
        self.device = self.storage.device

    def write_range(self, layer, block_ids, token_offset, key, value, *, validate=True) -> None:
        """Write ``[tokens, kv_heads, head_dim]`` rows at logical positions ``token_offset...`` of a page list."""
        self._check_layer(layer)
        if key.ndim != 3 or key.shape != value.shape:
            raise ValueError("key and value must both have shape [tokens, kv_heads, head_dim]")
        ids = _page_tensor(block_ids, self.shape, self.device)
        self._check_range(ids, token_offset, key.shape[0])
        write_kv_cache(self.key[layer], self.value[layer], ids, token_offset, key, value, self.shape.block_size,
                       validate=validate)

    def copy_blocks(self, pairs) -> None:
        """Apply copy-on-write ``(src, dst)`` page pairs to every layer of both pools."""
        copy_blocks(self.key, self.value, pairs)


class FP8KVCachePool(_Pool):
    """FP8 paged KV pool: the layout of :class:`PagedKVPool` with one byte per element.

    ``key``/``value`` are uint8 ``[layers, num_blocks, block_size, kv_heads,
    head_dim]`` tensors of OCP FP8 codes (``kv_format`` "e4m3" or "e5m2") with one
    fp32 scale for keys and one for values: an element ``x`` is stored as
    ``fp8(x * (1/scale))`` and read as ``code * scale``.  It holds twice the tokens
    of a bf16 pool in the same memory.  The reference has no FP8 pool;
    :meth:`attend` runs the decode attention of one layer.
    """

    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_dim, *, k_scale, v_scale,
                 kv_format="e4m3", device="cuda"):
        from ..kernels.fp8 import FORMATS, _scale

        self.shape = _geometry((num_layers, num_blocks, block_size, num_kv_heads, head_dim))
        if kv_format not in FORMATS:
            raise ValueError("kv_format must be 'e4m3' or 'e5m2'")
        if int(head_dim) % 2:
            raise ValueError("an fp8 pool needs an even head_dim (copy-on-write moves 16-bit words)")
        self.kv_format = kv_format
        self.k_scale, self.v_scale = _scale(k_scale, "k_scale"), _scale(v_scale, "v_scale")
        self.storage = torch.zeros((2, num_layers, num_blocks, block_size, num_kv_heads, head_dim),
                                   dtype=torch.uint8, device=device)
        self.key, self.value = self.storage[0], self.storage[1]
        self.device = self.storage.device

    def write_slots(self, layer, slot_mapping, key, value, *, validate=True) -> None:
        """Quantise ``key``/``value`` ``[tokens, kv_heads, head_dim]`` into rows ``slot_mapping`` of a layer."""
        from ..kernels.fp8 import write_kv_cache_slots_fp8

        self._check_layer(layer)
        write_kv_cache_slots_fp8(self.key[layer], self.value[layer], slot_mapping, key, value, self.k_scale,
                                 self.v_scale, kv_format=self.kv_format, validate=validate)

    def write_range(self, layer, block_ids, token_offset, key, value, *, validate=True) -> None:
        """Quantise a contiguous token range across pages; the slots are computed on the device."""
        if key.ndim != 3 or key.shape != value.shape:
            raise ValueError("key and value must both have shape [tokens, kv_heads, head_dim]")
        self._check_layer(layer)
        ids = _page_tensor(block_ids, self.shape, self.device)
        self._check_range(ids, token_offset, key.shape[0])
        if key.device != self.device or value.device != self.device:
            raise ValueError("CUDA KV write inputs must be on the cache device")
        bs = self.shape.block_size
        positions = torch.arange(key.shape[0], device=self.device, dtype=torch.long) + int(token_offset)
        self.write_slots(layer, ids[positions // bs] * bs + positions % bs, key, value, validate=False)

    def attend(self, layer, query, block_tables, context_lens, *, validate=True, workspace=None):
        """Decode attention of one layer over this pool (``paged_attention_fp8``)."""
        from ..kernels.fp8 import paged_attention_fp8

        self._check_layer(layer)
        return paged_attention_fp8(query, self.key[layer], self.value[layer], block_tables, context_lens,
                                   self.shape.block_size, self.k_scale, self.v_scale, kv_format=self.kv_format,
                                   validate=validate, workspace=workspace)

    def dequantized(self, layer, block_ids, token_count, dtype=torch.float32):
        """The first ``token_count`` logical rows of a page list, dequantised: ``(key, value)``."""
        self._check_layer(layer)
        ids = _page_tensor(block_ids, self.shape, self.device)
        if not 0 <= token_count <= ids.numel() * self.shape.block_size:
            raise ValueError("token_count must lie within the supplied block table capacity")
        fp8 = torch.float8_e4m3fn if self.kv_format == "e4m3" else torch.float8_e5m2
        out = []
        for codes, scale in ((self.key[layer], self.k_scale), (self.value[layer], self.v_scale)):
            rows = codes.index_select(0, ids).view(-1, self.shape.num_kv_heads, self.shape.head_dim)
            out.append(rows[:token_count].view(fp8).to(dtype) * scale)
        return tuple(out)

    def copy_blocks(self, pairs) -> None:
        """Apply copy-on-write ``(src, dst)`` pairs to every layer of both pools (16-bit word moves)."""
        copy_blocks(self.key.view(torch.bfloat16), self.value.view(torch.bfloat16), pairs)
