"""CPU oracle: paged decode attention.  Test infrastructure only (see oracle/__init__).

Restates
  * ``mini_engine/kernels/fallback.py:27-64``  (``paged_attention``, the torch
    decode path selected by ``backend="torch"`` in ``kernels/paged.py:10-11``);
  * ``benchmarks/compare_paged_backends.py:58-72`` (``fp32_oracle``: the same
    computation returned in fp32);
  * the *trusted-mode* guard semantics of the reference CUDA kernel
    ``mini_engine/kernels/csrc/paged_attention.cu:62-83, 99-121``: a token whose
    page id is outside ``[0, num_blocks)`` gets score -inf, an out-of-range
    context length (``<= 0`` or ``> table_width * block_size``) yields an
    all-zero row, and a row whose every token is masked yields zeros.
"""

from __future__ import annotations

import math

import torch


def _check(query, key_cache, value_cache, block_size):
    # fallback.py:42-47
    if query.ndim != 3 or key_cache.ndim != 4 or key_cache.shape != value_cache.shape:
        raise ValueError("invalid query or cache shape")
    if key_cache.shape[1] != block_size or query.shape[-1] != key_cache.shape[-1]:
        raise ValueError("block size or head dimension mismatch")
    if query.shape[1] % key_cache.shape[2]:
        raise ValueError("query heads must be divisible by KV heads")


def paged_attention_fp32(query, key_cache, value_cache, block_tables, context_lens, block_size, acc=torch.float32):
    """fp32 result of decode attention over each request's pages.

    ``query [B,Hq,D]``, caches ``[num_blocks, block_size, Hkv, D]``,
    ``block_tables [B, W]`` int64, ``context_lens [B]`` int64.  Raises
    ValueError("invalid context length") like fallback.py:50-52.  ``acc``
    (test control only) evaluates the same formula in another precision.
    """
    _check(query, key_cache, value_cache, block_size)
    scale = 1.0 / math.sqrt(query.shape[-1])  # fallback.py:48
    lengths = context_lens.cpu().tolist()
    tables = block_tables.cpu()
    outputs = []
    for batch, length in enumerate(lengths):  # fallback.py:49-63
        length = int(length)
        if length <= 0 or length > tables.shape[1] * block_size:
            raise ValueError("invalid context length")
        ids = tables[batch, : math.ceil(length / block_size)]
        keys = key_cache[ids].reshape(-1, key_cache.shape[2], key_cache.shape[3])[:length]
        values = value_cache[ids].reshape(-1, value_cache.shape[2], value_cache.shape[3])[:length]
        group = query.shape[1] // keys.shape[1]
        keys = keys.to(acc).repeat_interleave(group, dim=1)
        values = values.to(acc).repeat_interleave(group, dim=1)
        scores = torch.einsum("hd,thd->ht", query[batch].to(acc), keys) * scale
        probs = torch.softmax(scores, dim=-1)
        outputs.append(torch.einsum("ht,thd->hd", probs, values))
    return torch.stack(outputs)


def paged_attention(query, key_cache, value_cache, block_tables, context_lens, block_size):
    """Reference-dtype result (fallback.py:63: ``.to(query.dtype)``)."""
    return paged_attention_fp32(query, key_cache, value_cache, block_tables,
                                context_lens, block_size).to(query.dtype)


def paged_attention_fp64(query, key_cache, value_cache, block_tables, context_lens, block_size):
    """The same formula evaluated in float64, rounded to the query dtype.

    Not a reference path: a control that shows how far two valid evaluation
    orders of the reference's own formula move a model's outputs.
    """
    return paged_attention_fp32(query, key_cache, value_cache, block_tables, context_lens, block_size,
                                acc=torch.float64).to(query.dtype)


def paged_attention_trusted_fp32(query, key_cache, value_cache, block_tables, context_lens, block_size):
    """fp32 decode attention with the reference CUDA kernel's trusted-mode guards.

    paged_attention.cu:62-64 (count = 0 for an invalid length), :72-82
    (invalid page -> score -inf), :99/:120 (sum == 0 -> output 0).
    """
    _check(query, key_cache, value_cache, block_size)
    num_blocks = key_cache.shape[0]
    width = block_tables.shape[1]
    scale = 1.0 / math.sqrt(query.shape[-1])
    group = query.shape[1] // key_cache.shape[2]
    out = torch.zeros(query.shape, dtype=torch.float32)
    tables = block_tables.cpu()
    for batch, length in enumerate(context_lens.cpu().tolist()):
        length = int(length)
        if length <= 0 or length > width * block_size:
            continue
        tokens = torch.arange(length)
        pages = tables[batch, tokens // block_size]
        valid = (pages >= 0) & (pages < num_blocks)
        if not bool(valid.any()):
            continue
        safe = torch.where(valid, pages, torch.zeros_like(pages))
        keys = key_cache[safe, tokens % block_size].float().repeat_interleave(group, dim=1)
        values = value_cache[safe, tokens % block_size].float().repeat_interleave(group, dim=1)
        scores = torch.einsum("hd,thd->ht", query[batch].float(), keys) * scale
        scores = scores.masked_fill(~valid[None, :], float("-inf"))
        probs = torch.softmax(scores, dim=-1)
        out[batch] = torch.einsum("ht,thd->hd", probs, values)
    return out
