"""CPU oracle: ragged (packed) paged prefill attention.  Test infrastructure only.

Restates
  * ``mini_engine/kernels/prefill.py:61-131`` -- ``paged_prefill_attention``:
    the argument checks at :70-104 and the torch path at :114-131 (per request:
    gather pages, GQA repeat, fp32 SDPA with the absolute-position causal mask
    ``key <= start + i``);
  * ``tests/test_ragged_kernels.py:27-38`` -- the per-token fp32 oracle used by
    the reference's own CUDA tests.
Both compute in fp32; ``*_fp32`` variants return fp32, the others round to the
query dtype as prefill.py:130 does.
"""

from __future__ import annotations

import torch
from torch.nn import functional as F


def check_arguments(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables,
                    context_lens, block_size, *, validate=True):
    """The ValueError contract of prefill.py:70-104 (messages kept verbatim)."""
    if (type(block_size) is not int or block_size <= 0 or key_cache.ndim != 4
            or value_cache.shape != key_cache.shape or key_cache.shape[1] != block_size
            or any(size <= 0 for size in key_cache.shape)
            or not key_cache.is_contiguous() or not value_cache.is_contiguous()):
        raise ValueError("paged prefill caches must be contiguous [pages, block_size, kv_heads, head_dim]")
    if (q.ndim != 3 or q.shape[1] <= 0 or q.shape[2] != key_cache.shape[3]
            or q.shape[1] % key_cache.shape[2]):
        raise ValueError("paged prefill Q must be [tokens, heads, head_dim] with divisible GQA heads")
    if q.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError("paged prefill requires FP32/FP16/BF16")
    if key_cache.dtype != q.dtype or value_cache.dtype != q.dtype:
        raise ValueError("paged prefill Q/K/V must share dtype")
    metadata = (cu_seqlens_q, query_starts, block_tables, context_lens)
    if (cu_seqlens_q.ndim != 1 or query_starts.ndim != 1 or context_lens.ndim != 1
            or block_tables.ndim != 2 or query_starts.numel() != block_tables.shape[0]
            or context_lens.numel() != block_tables.shape[0]
            or cu_seqlens_q.numel() != block_tables.shape[0] + 1):
        raise ValueError("paged prefill metadata shapes do not match request count")
    if any(t.dtype != torch.int64 or not t.is_contiguous() for t in metadata):
        raise ValueError("paged prefill metadata must be contiguous int64 tensors")
    if any(t.device != q.device for t in (key_cache, value_cache, *metadata)):
        raise ValueError("paged prefill tensors must share device")
    if validate:
        offsets, starts, tables, lengths = (t.tolist() for t in metadata)
        if offsets[0] != 0 or offsets[-1] != q.shape[0] or any(b < a for a, b in zip(offsets, offsets[1:])):
            raise ValueError("query offsets must be monotone and cover all packed queries")
        for index, (start, length, table) in enumerate(zip(starts, lengths, tables)):
            count = offsets[index + 1] - offsets[index]
            if start < 0 or length != start + count or length > len(table) * block_size:
                raise ValueError("query start/context length exceeds block table capacity or query range")
            used = (length + block_size - 1) // block_size
            if any(page < 0 or page >= key_cache.shape[0] for page in table[:used]):
                raise ValueError("active block table contains an invalid physical page")


def paged_prefill_fp32(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables,
                       context_lens, block_size):
    """fp32 output of the torch path, prefill.py:114-131 (no argument checks)."""
    output = torch.zeros(q.shape, dtype=torch.float32)
    offsets, starts, lengths = (t.tolist() for t in (cu_seqlens_q, query_starts, context_lens))
    for index, (start, length) in enumerate(zip(starts, lengths)):
        begin, end = offsets[index:index + 2]
        if begin == end:
            continue
        pages = block_tables[index, :(length + block_size - 1) // block_size]
        key = key_cache[pages].reshape(-1, *key_cache.shape[2:])[:length]
        value = value_cache[pages].reshape(-1, *value_cache.shape[2:])[:length]
        groups = q.shape[1] // key.shape[1]
        key = key.repeat_interleave(groups, dim=1).transpose(0, 1).float()
        value = value.repeat_interleave(groups, dim=1).transpose(0, 1).float()
        query = q[begin:end].transpose(0, 1).float()
        mask = torch.arange(length)[None, :] <= (start + torch.arange(end - begin)[:, None])
        rows = F.scaled_dot_product_attention(query, key, value, attn_mask=mask)
        output[begin:end] = rows.transpose(0, 1)
    return output


def paged_prefill_attention(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables,
                            context_lens, block_size, *, validate=True):
    """prefill.py:61-131 with ``backend="torch"``: checks, then the fp32 path rounded to q's dtype."""
    check_arguments(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables,
                    context_lens, block_size, validate=validate)
    return paged_prefill_fp32(q, key_cache, value_cache, cu_seqlens_q, query_starts,
                              block_tables, context_lens, block_size).to(q.dtype)


def per_token_fp32(q, kc, vc, offsets, starts, tables, lengths, block):
    """Per packed token, attend keys ``[0, start + i]`` (tests/test_ragged_kernels.py:27-38)."""
    result = []
    offs = offsets.tolist()
    for request, (begin, end) in enumerate(zip(offs, offs[1:])):
        for token in range(begin, end):
            context = int(starts[request]) + token - begin + 1
            logical = torch.arange(context)
            physical = tables[request, logical // block]
            group = q.shape[1] // kc.shape[2]
            key = kc[physical, logical % block].repeat_interleave(group, dim=1).float()
            value = vc[physical, logical % block].repeat_interleave(group, dim=1).float()
            score = torch.einsum("hd,thd->ht", q[token].float(), key) / q.shape[-1] ** 0.5
            result.append(torch.einsum("ht,thd->hd", score.softmax(-1), value))
    if not result:
        return torch.zeros(q.shape, dtype=torch.float32)
    return torch.stack(result)
