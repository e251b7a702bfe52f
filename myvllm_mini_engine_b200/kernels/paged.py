"""Paged decode attention -- drop-in for ``mini_engine/kernels/paged.py``.

Same signature as the reference (paged.py:8-22).  There is one implementation,
the sm_100a split-KV kernel in libminikv; ``backend`` is accepted for
compatibility and must name a CUDA backend ("cuda", "cuda_baseline" and
"cuda_vector128" all run the same kernel).  Argument errors raise RuntimeError
with the messages of the reference's native checks
(``mini_engine/kernels/csrc/bindings.cpp:152-184``); ``validate=True`` adds the
same host-synchronising metadata checks (bindings.cpp:175-182).  fp32 is
supported in addition to fp16/bf16.
"""

from __future__ import annotations

import torch

from .. import _lib

CUDA_BACKENDS = ("cuda", "cuda_baseline", "cuda_vector128")
HEAD_DIMS = (16, 32, 64, 80, 96, 128, 192, 256)


def _require(condition, message):
    if not condition:
        raise RuntimeError(message)


def check_backend(backend):
    if backend not in CUDA_BACKENDS:
        raise ValueError("decode backend must be cuda, cuda_baseline or cuda_vector128 "
                         "(this package has no torch/CPU path)")


def paged_attention(query, key_cache, value_cache, block_tables, context_lens, block_size,
                    *, backend="cuda", validate=True, workspace=None, chained=False):
    """Decode attention ``out[b, h] = softmax(q . K^T / sqrt(D)) V`` over paged K/V.

    ``query [B, Hq, D]``, ``key_cache``/``value_cache`` ``[num_blocks, block_size,
    Hkv, D]``, ``block_tables [B, W]`` int64 (-1 padded), ``context_lens [B]`` int64.
    Returns a new ``[B, Hq, D]`` tensor in the query dtype.  ``workspace`` (a
    zero-filled uint8 CUDA tensor of at least :func:`workspace_bytes` bytes,
    reused as is by calls that do not overlap) may be passed; by default each
    stream gets a buffer kept by this module (see :func:`_workspace`).  Before
    capturing a CUDA graph, make one call on the capture stream so the buffer
    exists and its zero fill stays out of the graph.

    ``chained=True`` (an extension) declares that ``context_lens`` and
    ``block_tables`` were written before the previous kernel on the stream
    started -- e.g. the KV append of the same step is that kernel -- so the
    launch overlaps its prologue with that kernel (``minikv_paged_decode_chained``).
    """
    check_backend(backend)
    return _decode(query, key_cache, value_cache, block_tables, context_lens, block_size, validate=validate,
                   workspace=workspace, chained=chained)


def _decode(query, key_cache, value_cache, block_tables, context_lens, block_size, *, validate, workspace, chained,
            append=None):
    """Checks and launch of the decode; ``append = (key, value, token_offsets)`` selects the fused append."""
    _require(query.is_cuda, "query must be CUDA")
    for t in (key_cache, value_cache, block_tables, context_lens):
        _require(t.device == query.device, "all inputs must be on the same CUDA device")
        _require(t.is_contiguous(), "inputs must be contiguous")
    _require(query.is_contiguous(), "query must be contiguous")
    _require(query.dim() == 3 and key_cache.dim() == 4 and value_cache.shape == key_cache.shape,
             "invalid query/cache shapes")
    _require(query.dtype in _lib.DTYPE_CODES, "FP32/FP16/BF16 required")
    _require(key_cache.dtype == query.dtype and value_cache.dtype == query.dtype, "cache dtype mismatch")
    _require(block_tables.dtype == torch.int64 and context_lens.dtype == torch.int64, "metadata must be int64")
    batch, heads, dim = query.shape
    num_blocks, bs, kv_heads, _ = key_cache.shape
    _require(batch > 0 and heads > 0 and num_blocks > 0 and kv_heads > 0, "empty batch/heads/cache")
    _require(block_size > 0 and bs == block_size, "block size mismatch")
    _require(dim == key_cache.shape[3] and heads % kv_heads == 0, "head dimension or GQA mismatch")
    _require(dim in HEAD_DIMS, "supported head_dim: 16,32,64,80,96,128,192,256")
    _require(block_tables.dim() == 2 and block_tables.shape[0] == batch and block_tables.shape[1] > 0,
             "invalid block table")
    _require(context_lens.dim() == 1 and context_lens.shape[0] == batch, "invalid context lengths")
    width = block_tables.shape[1]
    _require(width * block_size <= 1048576, "maximum table capacity is 1M tokens")
    _require(batch * heads <= 2147483647, "batch/head product too large")
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
        need = lib.minikv_paged_decode_workspace_bytes(*key)
        if need < 0:
            _lib.check(_lib.EINVAL, "paged_attention")
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
            status = lib.minikv_paged_decode_append(
                query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_tables.data_ptr(),
                offsets.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(), workspace.data_ptr(),
                workspace.numel(), batch, heads, kv_heads, dim, num_blocks, block_size, width, code, int(chained),
                stream)
        else:
            entry = lib.minikv_paged_decode_chained if chained else lib.minikv_paged_decode
            status = entry(
                query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_tables.data_ptr(),
                context_lens.data_ptr(), out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                batch, heads, kv_heads, dim, num_blocks, block_size, width, code, stream)
    _lib.check(status, "paged_attention")
    return out


_WS_BYTES: dict = {}
_WORKSPACES: dict = {}
_RETIRED: list = []


def _workspace(device, stream, need):
    """Zero-filled scratch reused by every decode call on ``stream`` (a raw stream handle).

    The kernel keeps per-request ticket counters in it and leaves them at zero,
    so it is zeroed once, when allocated.  Calls on one stream never overlap;
    each stream gets its own buffer.  Buffers are never freed while the process
    runs, because a captured CUDA graph may still refer to one.
    """
    key = (device.index, stream)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < need:
        if buf is not None:
            _RETIRED.append(buf)
        buf = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf


def workspace_bytes(query, key_cache, block_tables):
    """Scratch bytes one :func:`paged_attention` call with these shapes needs."""
    lib = _lib.load()
    batch, heads, dim = query.shape
    num_blocks, block_size, kv_heads, _ = key_cache.shape
    need = lib.minikv_paged_decode_workspace_bytes(batch, heads, kv_heads, dim, num_blocks, block_size,
                                                   block_tables.shape[1], _lib.dtype_code(query.dtype))
    if need < 0:
        _lib.check(_lib.EINVAL, "workspace_bytes")
    return need


def paged_attention_with_append(query, key_cache, value_cache, block_tables, token_offsets, key, value, block_size,
                                *, backend="cuda", validate=True, workspace=None, chained=False):
    """KV append and decode attention in one launch (``minikv_paged_decode_append``).

    The same results as ``write_kv_cache_batch(key_cache, value_cache,
    block_tables, token_offsets, key, value, block_size)`` followed by
    ``paged_attention(query, key_cache, value_cache, block_tables,
    token_offsets + 1, block_size)`` -- the two calls of the reference's
    ``Attention.forward_decode_batch`` (``mini_engine/model/native_qwen3.py:188-196``)
    -- with one kernel: the CTA that attends a request's last tile writes the new
    K/V row into its pool slot (bit-exact) and reads it from ``key``/``value``.
    ``key``/``value`` are ``[B, Hkv, D]`` in the cache dtype.  ``validate=True``
    runs the checks of both calls.  Returns ``[B, Hq, D]``.  ``chained=True``:
    ``token_offsets``, ``block_tables`` and the pool rows the call reads (all but
    the appended ones) predate the previous kernel on the stream, while
    ``key``/``value`` may come from it; the launch then resolves its pages and
    starts staging pool rows while that kernel finishes.
    """
    check_backend(backend)
    _require(query.is_cuda, "query must be CUDA")
    _require(key.shape == value.shape and key.dim() == 3 and key.shape[0] == query.shape[0],
             "batch key/value must be [batch, kv_heads, head_dim]")
    for t in (key, value, token_offsets):
        _require(t.device == query.device and t.is_contiguous(), "batch KV write inputs must be contiguous CUDA tensors")
    _require(key.dtype == key_cache.dtype and value.dtype == key_cache.dtype, "batch KV dtype mismatch")
    _require(key_cache.dim() == 4 and key.shape[1:] == key_cache.shape[2:], "batch K/V shape mismatch")
    _require(token_offsets.dtype == torch.int64 and token_offsets.dim() == 1, "metadata must be int64")
    if validate:
        width = block_tables.shape[1] if block_tables.dim() == 2 else 0
        _require(not bool(((token_offsets < 0) | (token_offsets >= width * block_size)).any()),
                 "batch KV offset out of range")
    lengths = token_offsets + 1 if validate else token_offsets
    return _decode(query, key_cache, value_cache, block_tables, lengths, block_size, validate=validate,
                   workspace=workspace, chained=chained, append=(key, value, token_offsets))
