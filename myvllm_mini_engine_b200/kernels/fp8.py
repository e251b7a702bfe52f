"""FP8 KV pool (E4M3 or E5M2): quantising slot scatter and decode attention.

The reference has no FP8 KV pool (``VALIDATION_AND_BENCHMARKS.md:375`` lists it
as future work), so these two operators extend its API in its own style: the
scatter mirrors ``write_kv_cache_slots`` (``mini_engine/kernels/data.py:84-130``)
and the decode mirrors ``paged_attention`` (``kernels/paged.py:8-22``), each
with a key and a value scale.

A pool is a uint8 (or ``torch.float8_e4m3fn`` / ``torch.float8_e5m2``) tensor
of the 16-bit pool's shape ``[num_blocks, block_size, kv_heads, head_dim]``;
element ``x`` is stored as ``fp8(x * (1/scale))`` (fp32 product, nearest-even,
saturated to the largest finite code) and read as ``code * scale``.
``kv_format`` picks the byte format: "e4m3" (3 mantissa bits, range 448) or
"e5m2" (2 mantissa bits, range 57344, decoded with byte moves only, so its
decode runs faster).  A float8 pool dtype names its own format: ``kv_format``
may then be left as None, and a ``kv_format`` that contradicts it raises
ValueError.  A uint8 pool reads ``kv_format`` (None means "e4m3").  A decode step streams half the bytes of a bf16 pool.
"""

from __future__ import annotations

import torch

from .. import _lib
from .data import _backend, _rows
from .paged import _require, _workspace, check_backend
from .prefill import check_arguments

FP8_HEAD_DIMS = (32, 64, 96, 128, 192, 256)
_POOL_DTYPES = (torch.uint8, getattr(torch, "float8_e4m3fn", torch.uint8), getattr(torch, "float8_e5m2", torch.uint8))
FORMATS = {"e4m3": 0, "e5m2": 1}


_DTYPE_FORMATS = {dtype: name for dtype, name in ((getattr(torch, "float8_e4m3fn", None), "e4m3"),
                                                  (getattr(torch, "float8_e5m2", None), "e5m2")) if dtype is not None}


def _format(kv_format, pool_dtype=torch.uint8):
    """Format code of a pool: a float8 dtype decides it, a uint8 pool takes ``kv_format`` (default e4m3)."""
    if kv_format is not None and kv_format not in FORMATS:
        raise ValueError("kv_format must be 'e4m3' or 'e5m2'")
    implied = _DTYPE_FORMATS.get(pool_dtype)
    if implied is not None and kv_format not in (None, implied):
        raise ValueError(f"kv_format {kv_format!r} contradicts the {pool_dtype} pool")
    return FORMATS[implied or kv_format or "e4m3"]


def _scale(value, name):
    value = float(value)
    if not (value > 0.0 and value < float("inf")):
        raise ValueError(f"{name} must be finite and positive")
    return value


def write_kv_cache_slots_fp8(key_cache, value_cache, slot_mapping, key, value, k_scale, v_scale, *,
                             kv_format=None, backend="cuda", validate=True):
    """Quantise packed K/V rows into FP8 pools at ``slot_mapping`` (slots outside the capacity are skipped).

    ``key``/``value`` ``[tokens, kv_heads, head_dim]`` fp32/fp16/bf16 (token-strided
    views are read in place); pools ``[num_blocks, block_size, kv_heads, head_dim]``
    uint8 or a float8 dtype.  ``validate`` adds the host-synchronising slot checks
    of ``write_kv_cache_slots`` (data.py:109-119).
    """
    _backend(backend)
    fmt = _format(kv_format, key_cache.dtype)
    k_scale, v_scale = _scale(k_scale, "k_scale"), _scale(v_scale, "v_scale")
    if (key_cache.ndim != 4 or value_cache.shape != key_cache.shape
            or any(size <= 0 for size in key_cache.shape)
            or not key_cache.is_contiguous() or not value_cache.is_contiguous()):
        raise ValueError("KV caches must be contiguous [pages, block_size, kv_heads, head_dim]")
    if key_cache.dtype not in _POOL_DTYPES or value_cache.dtype != key_cache.dtype:
        raise ValueError("an fp8 KV pool must be uint8 or a float8 dtype")
    if key.ndim != 3 or key.shape != value.shape or key.shape[1:] != key_cache.shape[2:]:
        raise ValueError("packed key/value must be [tokens, kv_heads, head_dim] matching the cache")
    if key.dtype not in _lib.DTYPE_CODES or value.dtype != key.dtype:
        raise ValueError("packed KV requires FP32/FP16/BF16")
    if (slot_mapping.ndim != 1 or slot_mapping.numel() != key.shape[0]
            or slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous()):
        raise ValueError("slot_mapping must be contiguous int64 [tokens]")
    for tensor in (value_cache, slot_mapping, key, value):
        if tensor.device != key_cache.device:
            raise ValueError("packed KV tensors and slots must share the cache device")
    if (key_cache.shape[2] * key_cache.shape[3]) % 16:
        raise ValueError("fp8 KV row (kv_heads*head_dim) must be a multiple of 16")
    if validate:
        slots = slot_mapping.tolist()
        capacity = key_cache.shape[0] * key_cache.shape[1]
        if any(slot < 0 or slot >= capacity for slot in slots):
            raise ValueError("KV slot is outside cache capacity")
        if len(set(slots)) != len(slots):
            raise ValueError("duplicate KV slots would race during scatter")
    if key_cache.device.type != "cuda":
        raise ValueError("CUDA packed KV writes require CUDA tensors")
    tokens = key.shape[0]
    if tokens == 0:
        return
    # the kernel reads element by element: only the token stride must be uniform
    key, key_stride = _rows(key)
    value, value_stride = _rows(value)
    lib = _lib.load()
    with _lib.on_device(key_cache.device):
        status = lib.minikv_kv_scatter_slots_fp8(
            key_cache.data_ptr(), value_cache.data_ptr(), slot_mapping.data_ptr(), key.data_ptr(),
            value.data_ptr(), tokens, key_cache.shape[0], key_cache.shape[1], key_cache.shape[2],
            key_cache.shape[3], key_stride, value_stride, k_scale, v_scale, fmt, _lib.dtype_code(key.dtype),
            _lib.stream_of(key_cache.device))
    _lib.check(status, "write_kv_cache_slots_fp8")


_WS_BYTES: dict = {}


def paged_attention_fp8(query, key_cache, value_cache, block_tables, context_lens, block_size, k_scale, v_scale,
                        *, kv_format=None, backend="cuda", validate=True, workspace=None):
    """Decode attention over FP8 pools: ``softmax(q . (K*k_scale)^T / sqrt(D)) (V*v_scale)``.

    Arguments and guards as :func:`paged_attention` (``query [B, Hq, D]`` fp16 or
    bf16, ``block_tables [B, W]`` and ``context_lens [B]`` int64); the pools are
    uint8 or a float8 dtype holding ``kv_format`` codes.  Q.K and P.V run on fp16 tensor cores, so Q is
    rounded to fp16 (saturated at +-65504).  Returns ``[B, Hq, D]`` in the query dtype.
    """
    check_backend(backend)
    return _decode_fp8(query, key_cache, value_cache, block_tables, context_lens, block_size, k_scale, v_scale,
                       kv_format=kv_format, validate=validate, workspace=workspace)


def paged_attention_fp8_with_append(query, key_cache, value_cache, block_tables, token_offsets, key, value,
                                    block_size, k_scale, v_scale, *, kv_format=None, backend="cuda", validate=True,
                                    workspace=None, chained=False):
    """KV append and fp8 decode in one launch (``minikv_paged_decode_fp8_append``).

    The same results as quantising ``key``/``value`` ``[B, Hkv, D]`` (query dtype)
    into each request's slot for position ``token_offsets[b]`` with
    :func:`write_kv_cache_slots_fp8` and then :func:`paged_attention_fp8` over
    ``token_offsets + 1`` tokens: the CTA that attends a request's last tile
    quantises the new row into the pool (bit-exact with the scatter) and stages
    it from there.  The fp8 counterpart of
    :func:`~myvllm_mini_engine_b200.kernels.paged.paged_attention_with_append`,
    with the same ``chained`` contract.  Returns ``[B, Hq, D]``.
    """
    check_backend(backend)
    _require(query.is_cuda, "query must be CUDA")
    _require(key.shape == value.shape and key.dim() == 3 and key.shape[0] == query.shape[0],
             "batch key/value must be [batch, kv_heads, head_dim]")
    for t in (key, value, token_offsets):
        _require(t.device == query.device and t.is_contiguous(), "batch KV write inputs must be contiguous CUDA tensors")
    _require(key.dtype == query.dtype and value.dtype == query.dtype, "batch KV dtype must be the query dtype")
    _require(key_cache.dim() == 4 and key.shape[1:] == key_cache.shape[2:], "batch K/V shape mismatch")
    _require(token_offsets.dtype == torch.int64 and token_offsets.dim() == 1, "metadata must be int64")
    if validate:
        width = block_tables.shape[1] if block_tables.dim() == 2 else 0
        _require(not bool(((token_offsets < 0) | (token_offsets >= width * block_size)).any()),
                 "batch KV offset out of range")
    lengths = token_offsets + 1 if validate else token_offsets
    return _decode_fp8(query, key_cache, value_cache, block_tables, lengths, block_size, k_scale, v_scale,
                       kv_format=kv_format, validate=validate, workspace=workspace, chained=chained,
                       append=(key, value, token_offsets))


def _decode_fp8(query, key_cache, value_cache, block_tables, context_lens, block_size, k_scale, v_scale, *,
                kv_format, validate, workspace, chained=False, append=None):
    """Checks and launch of the fp8 decode; ``append = (key, value, token_offsets)`` selects the fused append."""
    fmt = _format(kv_format, key_cache.dtype)
    k_scale, v_scale = _scale(k_scale, "k_scale"), _scale(v_scale, "v_scale")
    _require(query.is_cuda, "query must be CUDA")
    for t in (key_cache, value_cache, block_tables, context_lens):
        _require(t.device == query.device, "all inputs must be on the same CUDA device")
        _require(t.is_contiguous(), "inputs must be contiguous")
    _require(query.is_contiguous(), "query must be contiguous")
    _require(query.dim() == 3 and key_cache.dim() == 4 and value_cache.shape == key_cache.shape,
             "invalid query/cache shapes")
    _require(query.dtype in (torch.float16, torch.bfloat16), "an fp8 KV pool needs an FP16/BF16 query")
    _require(key_cache.dtype in _POOL_DTYPES and value_cache.dtype == key_cache.dtype,
             "an fp8 KV pool must be uint8 or a float8 dtype")
    _require(block_tables.dtype == torch.int64 and context_lens.dtype == torch.int64, "metadata must be int64")
    batch, heads, dim = query.shape
    num_blocks, bs, kv_heads, _ = key_cache.shape
    _require(batch > 0 and heads > 0 and num_blocks > 0 and kv_heads > 0, "empty batch/heads/cache")
    _require(block_size > 0 and bs == block_size, "block size mismatch")
    _require(dim == key_cache.shape[3] and heads % kv_heads == 0, "head dimension or GQA mismatch")
    _require(dim in FP8_HEAD_DIMS, "fp8 KV pool: supported head_dim: 32,64,96,128,192,256")
    _require(block_tables.dim() == 2 and block_tables.shape[0] == batch and block_tables.shape[1] > 0,
             "invalid block table")
    _require(context_lens.dim() == 1 and context_lens.shape[0] == batch, "invalid context lengths")
    width = block_tables.shape[1]
    _require(width * block_size <= 1048576, "maximum table capacity is 1M tokens")
    if validate:
        _require(not bool(((context_lens <= 0) | (context_lens > width * block_size)).any()),
                 "invalid context length")
        positions = torch.arange(width, device=query.device, dtype=torch.int64) * block_size
        active = positions.unsqueeze(0) < context_lens.unsqueeze(1)
        _require(not bool((((block_tables < 0) | (block_tables >= num_blocks)) & active).any()),
                 "physical block id out of range")
    lib = _lib.load()
    code = _lib.dtype_code(query.dtype)
    key = (batch, heads, kv_heads, dim, num_blocks, block_size, width, code)
    need = _WS_BYTES.get(key)
    if need is None:
        need = lib.minikv_paged_decode_fp8_workspace_bytes(*key)
        if need < 0:
            _lib.check(_lib.EINVAL, "paged_attention_fp8")
        _WS_BYTES[key] = need
    with _lib.on_device(query.device):
        stream = _lib.stream_of(query.device)
        if workspace is None:
            workspace = _workspace(query.device, stream, need)
        elif workspace.numel() < need:
            raise RuntimeError("decode workspace too small")
        out = torch.empty_like(query)
        if append is not None:
            key, value, offsets = append
            status = lib.minikv_paged_decode_fp8_append(
                query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_tables.data_ptr(),
                offsets.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(), workspace.data_ptr(),
                workspace.numel(), batch, heads, kv_heads, dim, num_blocks, block_size, width, k_scale, v_scale,
                fmt, code, int(chained), stream)
        else:
            status = lib.minikv_paged_decode_fp8(
                query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_tables.data_ptr(),
                context_lens.data_ptr(), out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                batch, heads, kv_heads, dim, num_blocks, block_size, width, k_scale, v_scale, fmt, code, stream)
    _lib.check(status, "paged_attention_fp8")
    return out


def paged_prefill_attention_fp8(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens,
                                block_size, k_scale, v_scale, *, kv_format=None, backend="cuda", validate=True,
                                max_query_len=None):
    """Ragged causal prefill over FP8 pools: :func:`paged_prefill_attention` with K/V read as ``code * scale``.

    Arguments, checks and messages as ``paged_prefill_attention``
    (``mini_engine/kernels/prefill.py:61-131``), plus the pools' scales and
    format.  ``q`` is fp16 or bf16 ``[tokens, q_heads, head_dim]``.  On the
    tcgen05 prefill's shapes (GQA group dividing 128, block_size a multiple of
    8): at head_dim 128 the kernel stages the codes with TMA and converts them
    to fp16 in shared memory (a bf16 Q is rounded to fp16 for the products);
    at head_dim 64 it runs on a dense ``q.dtype`` copy of the pages the tables
    reference (codes converted exactly).  Either way the key scale is folded
    into the softmax scale and the value scale into the output.  Other shapes,
    and batches whose copy would pass 8 GiB, run each query token as one row of
    the fp8 split-KV decode kernel (the CUDA-core route; Q rounded to fp16 for
    the products).
    """
    if backend != "cuda":
        raise ValueError("paged prefill backend must be cuda (this package has no torch/CPU path)")
    fmt = _format(kv_format, key_cache.dtype)
    k_scale, v_scale = _scale(k_scale, "k_scale"), _scale(v_scale, "v_scale")
    check_arguments(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens, block_size,
                    validate, cache_dtypes=_POOL_DTYPES)
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("an fp8 KV pool needs an FP16/BF16 query")
    if q.device.type != "cuda":
        raise ValueError("CUDA paged prefill requires CUDA tensors")
    if q.shape[2] not in FP8_HEAD_DIMS:
        raise ValueError("fp8 KV pool: supported head_dim: 32,64,96,128,192,256")
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
    need = lib.minikv_paged_prefill_fp8_workspace_bytes(tokens, requests, q.shape[1], kv_heads, dim, num_blocks,
                                                        block_size, width, bound, code)
    if need < 0:
        _lib.check(_lib.EINVAL, "paged_prefill_attention_fp8")
    workspace = torch.empty(need, dtype=torch.uint8, device=q.device) if need > 0 else None  # 0: not read
    with _lib.on_device(q.device):
        status = lib.minikv_paged_prefill_fp8(
            q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), cu_seqlens_q.data_ptr(),
            query_starts.data_ptr(), block_tables.data_ptr(), context_lens.data_ptr(), output.data_ptr(),
            workspace.data_ptr() if need > 0 else None, need, tokens, requests, q.shape[1], kv_heads, dim, num_blocks,
            block_size, width, bound, k_scale, v_scale, fmt, code, _lib.stream_of(q.device))
    _lib.check(status, "paged_prefill_attention_fp8")
    return output
