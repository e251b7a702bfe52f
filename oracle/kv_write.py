"""CPU oracle: KV writes and copy-on-write.  Test infrastructure only (see oracle/__init__).

All functions are bit-exact byte moves done with numpy on raw integer views of
the (CPU) torch tensors, so fp32 / fp16 / bf16 are handled identically.

Restates
  * ``write_kv_cache``       -- ``mini_engine/kernels/data.py:39-64`` (torch path
    :51-62) with the CUDA guard semantics of ``csrc/data.cu:68-86``;
  * ``write_kv_cache_batch`` -- ``data.py:67-81`` and ``csrc/data.cu:89-107``
    (trusted mode: a request whose page index is outside the table or whose
    physical page is outside ``[0, num_blocks)`` writes nothing);
  * ``write_kv_cache_slots`` -- ``data.py:84-130`` (``index_copy_`` at :120-125)
    and ``csrc/data.cu:196-206`` (a slot outside the capacity writes nothing);
  * ``copy_blocks``          -- copy-on-write, which the reference does not have
    (the survey of ``block_manager.py:99-116`` found no CoW); its contract is the
    torch expression ``pool[:, dst] = pool[:, src]`` over all layers.
"""

from __future__ import annotations

import numpy as np
import torch

_RAW = {1: torch.int8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def raw(tensor: torch.Tensor) -> np.ndarray:
    """numpy view sharing memory with a CPU tensor, as same-width integers."""
    return tensor.view(_RAW[tensor.element_size()]).numpy()


def write_kv_cache(key_cache, value_cache, block_ids, token_offset, key, value, block_size):
    """Contiguous token range through one block list (data.py:51-62)."""
    kc, vc = raw(key_cache), raw(value_cache)
    k, v = raw(key.contiguous()), raw(value.contiguous())
    ids = np.asarray(block_ids.cpu().reshape(-1).tolist() if isinstance(block_ids, torch.Tensor)
                     else list(block_ids), dtype=np.int64)
    num_blocks = kc.shape[0]
    for token in range(k.shape[0]):  # data.cu:72-85 one token per CTA
        logical = token_offset + token
        index, slot = divmod(logical, block_size)
        if index < 0 or index >= ids.size:
            continue
        physical = int(ids[index])
        if physical < 0 or physical >= num_blocks:
            continue
        kc[physical, slot] = k[token]
        vc[physical, slot] = v[token]


def write_kv_cache_batch(key_cache, value_cache, block_tables, token_offsets, key, value, block_size):
    """One token per request at ``token_offsets[r]`` (data.py:76-80, data.cu:93-106)."""
    kc, vc = raw(key_cache), raw(value_cache)
    k, v = raw(key.contiguous()), raw(value.contiguous())
    tables = block_tables.cpu().numpy()
    offsets = token_offsets.cpu().numpy()
    num_blocks = kc.shape[0]
    for request in range(k.shape[0]):
        logical = int(offsets[request])
        index, slot = logical // block_size, logical % block_size
        if index < 0 or index >= tables.shape[1]:
            continue
        physical = int(tables[request, index])
        if physical < 0 or physical >= num_blocks:
            continue
        kc[physical, slot] = k[request]
        vc[physical, slot] = v[request]


def write_kv_cache_slots(key_cache, value_cache, slot_mapping, key, value):
    """Flat scatter ``rows[slot_mapping[t]] = key[t]`` (data.py:120-125)."""
    rows_k = raw(key_cache).reshape(-1, *key_cache.shape[2:])
    rows_v = raw(value_cache).reshape(-1, *value_cache.shape[2:])
    k, v = raw(key.contiguous()), raw(value.contiguous())
    slots = slot_mapping.cpu().numpy()
    capacity = rows_k.shape[0]
    keep = (slots >= 0) & (slots < capacity)  # data.cu:200-201
    rows_k[slots[keep]] = k[keep]
    rows_v[slots[keep]] = v[keep]


def copy_blocks(key_pool, value_pool, pairs):
    """Copy-on-write of whole pages across every layer: ``pool[:, dst] = pool[:, src]``.

    ``key_pool``/``value_pool`` are ``[layers, num_blocks, block_size, Hkv, D]``;
    ``pairs`` is a sequence of ``(src, dst)`` physical page ids.  Copies are
    applied in order, each reading the pool as left by the previous one.
    """
    kp, vp = raw(key_pool), raw(value_pool)
    for src, dst in pairs:
        kp[:, int(dst)] = kp[:, int(src)]
        vp[:, int(dst)] = vp[:, int(src)]
