"""Ragged paged prefill -- drop-in for ``paged_prefill_attention`` in
``mini_engine/kernels/prefill.py`` (:61-131).

Same signature, ValueError checks and messages as the reference (:70-104).
The CUDA path runs libminikv: tcgen05 tensor-core tiles for bf16/fp16 with
head_dim 64/128 and a GQA group dividing 128, a CUDA-core route otherwise
(fp32 included).  There is no torch path.
"""

from __future__ import annotations

import torch

from .. import _lib

HEAD_DIMS = (16, 32, 64, 80, 96, 128, 192, 256)


def check_arguments(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables,
                    context_lens, block_size, validate, cache_dtypes=None):
    """prefill.py:70-104.  ``cache_dtypes``: the caches' allowed dtypes when they differ from Q's (FP8 pools)."""
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
    if cache_dtypes is None and (key_cache.dtype != q.dtype or value_cache.dtype != q.dtype):
        raise ValueError("paged prefill Q/K/V must share dtype")
    if cache_dtypes is not None and (key_cache.dtype not in cache_dtypes or value_cache.dtype != key_cache.dtype):
        raise ValueError("an fp8 KV pool must be uint8 or a float8 dtype")
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


def paged_prefill_attention(q, key_cache, value_cache, cu_seqlens_q, query_starts,
                            block_tables, context_lens, block_size, *, backend="cuda", validate=True,
                            max_query_len=None):
    """Packed causal queries read paged KV directly (prefill.py:61-131).

    Q is ``[total_queries, query_heads, head_dim]``.  Each request describes a
    suffix starting at its absolute ``query_start``; ``context_len`` equals
    ``start + query_count``.  ``max_query_len`` (optional) is a host-side bound
    on any request's query count; it defaults to the number of packed tokens.
    """
    if backend != "cuda":
        raise ValueError("paged prefill backend must be cuda (this package has no torch/CPU path)")
    check_arguments(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables,
                    context_lens, block_size, validate)
    if q.device.type != "cuda":
        raise ValueError("CUDA paged prefill requires CUDA tensors")
    if q.shape[2] not in HEAD_DIMS:
        raise ValueError("CUDA paged prefill supports head_dim 16,32,64,80,96,128,192,256")
    q = q.contiguous()
    output = torch.empty_like(q)
    tokens = q.shape[0]
    if tokens == 0:
        return output
    requests = block_tables.shape[0]
    num_blocks, _, kv_heads, dim = key_cache.shape
    width = block_tables.shape[1]
    bound = tokens if max_query_len is None else int(max_query_len)
    lib = _lib.load()
    code = _lib.dtype_code(q.dtype)
    need = lib.minikv_paged_prefill_workspace_bytes(tokens, requests, q.shape[1], kv_heads, dim, num_blocks,
                                                    block_size, width, bound, code)
    if need < 0:
        _lib.check(_lib.EINVAL, "paged_prefill_attention")
    workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    with _lib.on_device(q.device):
        status = lib.minikv_paged_prefill(
            q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), cu_seqlens_q.data_ptr(),
            query_starts.data_ptr(), block_tables.data_ptr(), context_lens.data_ptr(), output.data_ptr(),
            workspace.data_ptr(), workspace.numel(), tokens, requests, q.shape[1], kv_heads, dim,
            num_blocks, block_size, width, bound, code, _lib.stream_of(q.device))
    _lib.check(status, "paged_prefill_attention")
    return output
