"""KV writes -- drop-in for the KV entry points of ``mini_engine/kernels/data.py``.

``write_kv_cache`` (data.py:39-64), ``write_kv_cache_batch`` (:67-81) and
``write_kv_cache_slots`` (:84-130) keep the reference signatures, ValueError
checks and messages; native argument errors raise RuntimeError as the
reference's TORCH_CHECKs do (bindings.cpp:110-150, data.cu:209-237).  All three
run the libminikv row-scatter kernel (bit-exact 16-byte copies); fp32 caches
are accepted too.  ``copy_blocks`` is new: the copy-on-write kernel used when a
request must write into a page that other requests still reference.
"""

from __future__ import annotations

import torch

from .. import _lib


def _backend(backend):
    # data.py:9-11, minus the torch path: this package has no CPU fallback.
    if backend != "cuda":
        raise ValueError("data backend must be cuda (this package has no torch/CPU path)")


def _require(condition, message):
    if not condition:
        raise RuntimeError(message)


def _as_long(tensor, device):
    """``tensor`` as a contiguous int64 tensor on ``device`` (itself when it already is one)."""
    if tensor.dtype == torch.long and tensor.device == device and tensor.is_contiguous():
        return tensor
    return tensor.to(device=device, dtype=torch.long).contiguous()


def _row_stride(tensor):
    """Token stride (elements) of a [tokens, Hkv, D] tensor whose rows are contiguous, else None."""
    if tensor.dim() != 3:
        return None
    _, heads, dim = tensor.shape
    if (dim > 1 and tensor.stride(2) != 1) or (heads > 1 and tensor.stride(1) != dim):
        return None
    return tensor.stride(0) if tensor.shape[0] > 1 else heads * dim


def _rows(tensor):
    """(tensor, token stride) with rows contiguous and 16-byte aligned, copying only if needed."""
    stride = _row_stride(tensor)
    if (stride is None or (stride * tensor.element_size()) % 16 or tensor.data_ptr() % 16
            or stride < tensor.shape[1] * tensor.shape[2]):
        tensor = tensor.contiguous()
        stride = tensor.shape[1] * tensor.shape[2]
    return tensor, stride


def write_kv_cache(key_cache, value_cache, block_ids, token_offset, key, value,
                   block_size, *, backend="cuda", validate=True):
    """Write a contiguous token range starting at ``token_offset`` through ``block_ids``."""
    _backend(backend)
    if key.shape != value.shape or key.ndim != 3:  # data.py:42-47
        raise ValueError("key and value must be [tokens, kv_heads, head_dim]")
    if key.device != key_cache.device or value.device != key_cache.device:
        raise ValueError("KV tensors must be on the cache device")
    if key.dtype != key_cache.dtype or value.dtype != key_cache.dtype:
        raise ValueError("KV tensors must match cache dtype")
    ids = block_ids.reshape(-1).to(device=key_cache.device, dtype=torch.long)  # :48
    if token_offset < 0 or token_offset + key.shape[0] > ids.numel() * block_size:
        raise ValueError("write exceeds supplied block table capacity")
    # bindings.cpp:113-124
    for t in (key_cache, value_cache, ids, key, value):
        _require(t.is_cuda and t.is_contiguous(), "KV write inputs must be contiguous CUDA tensors")
        _require(t.device == key_cache.device, "KV write inputs must share a device")
    _require(key_cache.dim() == 4 and value_cache.shape == key_cache.shape, "cache shape mismatch")
    _require(block_size > 0 and key_cache.shape[1] == block_size, "block size mismatch")
    _require(key.shape[1] == key_cache.shape[2] and key.shape[2] == key_cache.shape[3], "K/V head shape mismatch")
    _require(key_cache.dtype in _lib.DTYPE_CODES, "KV cache requires FP32/FP16/BF16")
    if validate:  # data.cu:169
        _require(not bool(((ids < 0) | (ids >= key_cache.shape[0])).any()), "KV physical block id out of range")
    tokens = key.shape[0]
    if tokens == 0:
        return
    lib = _lib.load()
    row = key.shape[1] * key.shape[2]
    with _lib.on_device(key_cache.device):
        status = lib.minikv_kv_write_range(
            key_cache.data_ptr(), value_cache.data_ptr(), ids.data_ptr(), ids.numel(), int(token_offset),
            key.data_ptr(), value.data_ptr(), tokens, key_cache.shape[0], block_size, key.shape[1], key.shape[2],
            row, row, _lib.dtype_code(key_cache.dtype), _lib.stream_of(key_cache.device))
    _lib.check(status, "write_kv_cache")


def write_kv_cache_batch(key_cache, value_cache, block_tables, token_offsets, key, value,
                         block_size, *, backend="cuda", validate=True):
    """Decode append: request ``r`` writes ``key[r]``/``value[r]`` at position ``token_offsets[r]``."""
    _backend(backend)
    if key.shape != value.shape or key.ndim != 3:  # data.py:70-74
        raise ValueError("batch key/value must be [batch, kv_heads, head_dim]")
    if (block_tables.ndim != 2 or token_offsets.ndim != 1 or block_tables.shape[0] != key.shape[0]
            or token_offsets.shape[0] != key.shape[0]):
        raise ValueError("batch block table or offset shape mismatch")
    tables = _as_long(block_tables, key_cache.device)
    offsets = _as_long(token_offsets, key_cache.device)
    for t in (key_cache, value_cache, tables, offsets, key, value):  # bindings.cpp:131-142
        _require(t.is_cuda and t.is_contiguous(), "batch KV write inputs must be contiguous CUDA tensors")
        _require(t.device == key_cache.device, "batch KV write inputs must share a device")
    _require(key_cache.dim() == 4 and value_cache.shape == key_cache.shape, "batch cache shape mismatch")
    _require(block_size > 0 and key_cache.shape[1] == block_size, "batch block size mismatch")
    _require(key.shape[1] == key_cache.shape[2] and key.shape[2] == key_cache.shape[3], "batch K/V shape mismatch")
    _require(key_cache.dtype in _lib.DTYPE_CODES, "batch KV cache requires FP32/FP16/BF16")
    _require(key.dtype == key_cache.dtype and value.dtype == key_cache.dtype, "batch KV dtype mismatch")
    if validate:  # bindings.cpp:143-148 and data.cu:179
        _require(not bool(((offsets < 0) | (offsets >= tables.shape[1] * block_size)).any()),
                 "batch KV offset out of range")
        _require(not bool(((tables < 0) | (tables >= key_cache.shape[0])).any()),
                 "KV batch physical block id out of range")
    batch = key.shape[0]
    if batch == 0:
        return
    lib = _lib.load()
    row = key.shape[1] * key.shape[2]
    with _lib.on_device(key_cache.device):
        status = lib.minikv_kv_append_batch(
            key_cache.data_ptr(), value_cache.data_ptr(), tables.data_ptr(), offsets.data_ptr(), key.data_ptr(),
            value.data_ptr(), batch, tables.shape[1], key_cache.shape[0], block_size, key.shape[1], key.shape[2],
            row, row, _lib.dtype_code(key_cache.dtype), _lib.stream_of(key_cache.device))
    _lib.check(status, "write_kv_cache_batch")


def write_kv_cache_slots(key_cache, value_cache, slot_mapping, key, value, *, backend="cuda", validate=True):
    """Scatter packed KV rows to unique physical ``page * block_size + offset`` slots.

    ``validate=False`` trusts slot contents checked by the batch factory; shape,
    dtype, device and cache layout checks remain active without a device sync
    (data.py:84-130).  Key/value may be token-strided views (split projection
    outputs); their rows are read in place.
    """
    _backend(backend)
    if (key_cache.ndim != 4 or value_cache.shape != key_cache.shape
            or any(size <= 0 for size in key_cache.shape)
            or not key_cache.is_contiguous() or not value_cache.is_contiguous()):
        raise ValueError("KV caches must be contiguous [pages, block_size, kv_heads, head_dim]")
    if key.ndim != 3 or key.shape != value.shape or key.shape[1:] != key_cache.shape[2:]:
        raise ValueError("packed key/value must be [tokens, kv_heads, head_dim] matching the cache")
    if (slot_mapping.ndim != 1 or slot_mapping.numel() != key.shape[0]
            or slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous()):
        raise ValueError("slot_mapping must be contiguous int64 [tokens]")
    for tensor in (value_cache, slot_mapping, key, value):
        if tensor.device != key_cache.device:
            raise ValueError("packed KV tensors and slots must share the cache device")
    if any(t.dtype != key_cache.dtype for t in (value_cache, key, value)):
        raise ValueError("packed KV tensors must share the cache dtype")
    if key_cache.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError("packed KV requires FP32/FP16/BF16")
    if validate:  # data.py:109-119
        slots = slot_mapping.tolist()
        capacity = key_cache.shape[0] * key_cache.shape[1]
        if any(slot < 0 or slot >= capacity for slot in slots):
            raise ValueError("KV slot is outside cache capacity")
        if len(set(slots)) != len(slots):
            raise ValueError("duplicate KV slots would race during scatter")
        if (torch._C._overlaps(key_cache, value_cache)
                or any(torch._C._overlaps(cache, source)
                       for cache in (key_cache, value_cache) for source in (key, value, slot_mapping))):
            raise ValueError("KV destinations and source tensors must not overlap")
    if key_cache.device.type != "cuda":
        raise ValueError("CUDA packed KV writes require CUDA tensors")
    tokens = key.shape[0]
    if tokens == 0:
        return
    key, key_stride = _rows(key)
    value, value_stride = _rows(value)
    lib = _lib.load()
    with _lib.on_device(key_cache.device):
        status = lib.minikv_kv_scatter_slots(
            key_cache.data_ptr(), value_cache.data_ptr(), slot_mapping.data_ptr(), key.data_ptr(),
            value.data_ptr(), tokens, key_cache.shape[0], key_cache.shape[1], key_cache.shape[2],
            key_cache.shape[3], key_stride, value_stride, _lib.dtype_code(key_cache.dtype),
            _lib.stream_of(key_cache.device))
    _lib.check(status, "write_kv_cache_slots")


def copy_blocks(key_pool, value_pool, pairs, *, validate=True):
    """Copy-on-write: ``pool[:, dst] = pool[:, src]`` for each ``(src, dst)`` in ``pairs``.

    ``key_pool``/``value_pool`` are the full ``[layers, num_blocks, block_size,
    Hkv, D]`` pools; ``pairs`` is an int64 ``[n, 2]`` tensor on the pool device
    or a sequence of pairs (copied to the device).  Destinations must be
    distinct and must not be used as a source by another pair.
    """
    if key_pool.ndim != 5 or value_pool.shape != key_pool.shape:
        raise ValueError("KV pools must be [layers, pages, block_size, kv_heads, head_dim]")
    if not key_pool.is_contiguous() or not value_pool.is_contiguous() or not key_pool.is_cuda:
        raise ValueError("KV pools must be contiguous CUDA tensors")
    if key_pool.dtype not in _lib.DTYPE_CODES or value_pool.dtype != key_pool.dtype:
        raise ValueError("KV pools must share an FP32/FP16/BF16 dtype")
    if not isinstance(pairs, torch.Tensor):
        pairs = torch.tensor([[int(s), int(d)] for s, d in pairs], dtype=torch.int64).reshape(-1, 2)
    if pairs.ndim != 2 or pairs.shape[1] != 2 or pairs.dtype != torch.int64:
        raise ValueError("pairs must be int64 [n, 2] (src, dst)")
    if validate:
        host = pairs.cpu().tolist()
        dsts = [d for _, d in host]
        if any(not (0 <= v < key_pool.shape[1]) for pair in host for v in pair):
            raise ValueError("copy-on-write page id out of range")
        if len(set(dsts)) != len(dsts) or set(dsts) & {s for s, _ in host}:
            raise ValueError("copy-on-write destinations must be distinct and never a source")
    pairs = pairs.to(key_pool.device).contiguous()
    if pairs.shape[0] == 0:
        return
    lib = _lib.load()
    layers, num_blocks = key_pool.shape[:2]
    block_elems = key_pool[0, 0].numel()
    with _lib.on_device(key_pool.device):
        status = lib.minikv_copy_blocks(key_pool.data_ptr(), value_pool.data_ptr(), pairs.data_ptr(),
                                        pairs.shape[0], layers, num_blocks, block_elems,
                                        _lib.dtype_code(key_pool.dtype), _lib.stream_of(key_pool.device))
    _lib.check(status, "copy_blocks")
