"""Seeded synthetic cases for the paged-KV hot path (inputs only).

Every case is built from ``numpy.random.Generator(PCG64(seed))`` so the same
bytes come out on the build container and on the GPU box.  Shapes follow the
five BASELINE configurations and the reference's own test fixtures
(``tests/test_cuda_paged_attention.py:17-26``, ``tests/test_ragged_kernels.py:17-24``,
``tests/test_data_kernels.py:41-57``, ``tests/test_ragged_model.py:42-53``).

``make_golden.py`` feeds these inputs to the reference's torch paths and stores
the outputs; the tests rebuild the inputs, check ``inputs_sha256`` and compare.
Tensors are CPU tensors; tests move them to the GPU.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np
import torch

HQ, HKV, D = 16, 8, 128


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def randn(gen, shape, dtype):
    return torch.from_numpy(gen.standard_normal(size=shape, dtype=np.float32)).to(dtype)


def sha256_of(tensors):
    digest = hashlib.sha256()
    for tensor in tensors:
        t = tensor.contiguous()
        digest.update(str((tuple(t.shape), str(t.dtype))).encode())
        digest.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return digest.hexdigest()


# --------------------------------------------------------------------------- decode

def decode_case(dtype, *, head_dim=D, block_size=16, lengths=(17, 257, 521), heads=HQ,
                kv_heads=HKV, seed=23, spare=3):
    """Decode attention inputs shaped like test_cuda_paged_attention.py:17-26.

    Pages come from a seeded permutation of the pool, so tables are
    non-contiguous; ``spare`` unused pages stay in the pool.
    """
    gen = rng(seed)
    width = (max(lengths) + block_size - 1) // block_size
    blocks = len(lengths) * width + spare
    key = randn(gen, (blocks, block_size, kv_heads, head_dim), dtype)
    value = randn(gen, (blocks, block_size, kv_heads, head_dim), dtype)
    table = torch.from_numpy(gen.permutation(blocks)[:len(lengths) * width].astype(np.int64))
    table = table.view(len(lengths), width)
    lens = torch.tensor(lengths, dtype=torch.int64)
    query = randn(gen, (len(lengths), heads, head_dim), dtype)
    return {"query": query, "key_cache": key, "value_cache": value, "block_tables": table,
            "context_lens": lens, "block_size": block_size}


def append_decode_case(dtype, *, batch, contexts, block_size, pool_blocks=None, seed,
                       heads=HQ, kv_heads=HKV, head_dim=D, pool_slack=1.1):
    """One decode step of BASELINE configs 1-3: append K/V at ``contexts[b]``, attend ``contexts[b]+1``.

    The pool holds random N(0,1) history; each request's pages are a slice of a
    seeded permutation of the whole pool (non-contiguous).  With
    ``pool_blocks=None`` the pool is sized to ``pool_slack`` x the pages used.
    """
    gen = rng(seed)
    contexts = [int(c) for c in contexts]
    pages = [(c + 1 + block_size - 1) // block_size for c in contexts]
    width = max(pages)
    if pool_blocks is None:
        pool_blocks = math.ceil(pool_slack * sum(pages))
    if pool_blocks < sum(pages):
        raise ValueError("pool too small for the case")
    perm = gen.permutation(pool_blocks).astype(np.int64)
    table = np.full((batch, width), -1, dtype=np.int64)
    cursor = 0
    for b, count in enumerate(pages):
        table[b, :count] = perm[cursor:cursor + count]
        cursor += count
    key_cache = randn(gen, (pool_blocks, block_size, kv_heads, head_dim), dtype)
    value_cache = randn(gen, (pool_blocks, block_size, kv_heads, head_dim), dtype)
    query = randn(gen, (batch, heads, head_dim), dtype)
    new_key = randn(gen, (batch, kv_heads, head_dim), dtype)
    new_value = randn(gen, (batch, kv_heads, head_dim), dtype)
    offsets = torch.tensor(contexts, dtype=torch.int64)
    return {"query": query, "key_cache": key_cache, "value_cache": value_cache,
            "block_tables": torch.from_numpy(table), "token_offsets": offsets,
            "key": new_key, "value": new_value, "context_lens": offsets + 1,
            "block_size": block_size}


def config1():
    """fp32, B1, context 128, bs16, pool of 64 blocks; append at 128, attend 129."""
    return append_decode_case(torch.float32, batch=1, contexts=[128], block_size=16,
                              pool_blocks=64, seed=101)


def config2():
    """fp16, B8, every context 512, bs256, pool of 64 blocks (24 used)."""
    return append_decode_case(torch.float16, batch=8, contexts=[512] * 8, block_size=256,
                              pool_blocks=64, seed=102)


def config3_lengths(seed=103, batch=32):
    return [int(x) for x in rng(seed + 1000).integers(1, 2049, size=batch)]


def config3():
    """bf16, B32, contexts U[1,2048] seeded, bs16, pool = 1.1 x pages used."""
    return append_decode_case(torch.bfloat16, batch=32, contexts=config3_lengths(),
                              block_size=16, seed=103)


def headline_case(batch=32, context=2048, seed=104):
    """B32 x ctx2048 (attended, after the append), bf16, bs16 -- the north-star shape."""
    return append_decode_case(torch.bfloat16, batch=batch, contexts=[context - 1] * batch,
                              block_size=16, seed=seed)


# --------------------------------------------------------------------------- KV writes

def slots_case(dtype=torch.float32, dim=16, seed=631):
    """Cache/slots of tests/test_ragged_kernels.py:17-24, 48-65 (8 pages x 4 slots x 2 heads)."""
    gen = rng(seed)
    key = randn(gen, (8, 4, 2, dim), dtype)
    value = randn(gen, (8, 4, 2, dim), dtype)
    packed = randn(gen, (8, 4, dim), dtype)
    slots = torch.tensor([5, 6, 7, 9, 10, 11, 28, 29], dtype=torch.int64)
    return {"key_cache": key, "value_cache": value, "slot_mapping": slots,
            "key": packed[:, :2], "value": packed[:, 2:]}


def range_case(dtype=torch.float16, seed=63):
    """tests/test_data_kernels.py:41-57: 7 tokens from offset 1 across pages [4, 1, 5]."""
    gen = rng(seed)
    block_size, blocks, kv_heads, dim = 4, 6, 2, 8
    return {"key_cache": torch.zeros(blocks, block_size, kv_heads, dim, dtype=dtype),
            "value_cache": torch.zeros(blocks, block_size, kv_heads, dim, dtype=dtype),
            "block_ids": torch.tensor([4, 1, 5], dtype=torch.int64), "token_offset": 1,
            "key": randn(gen, (7, kv_heads, dim), dtype), "value": randn(gen, (7, kv_heads, dim), dtype),
            "block_size": block_size}


def batch_write_case(dtype=torch.bfloat16, seed=64):
    """Decode append for 5 requests, two of which point at invalid pages (trusted mode)."""
    gen = rng(seed)
    block_size, blocks, kv_heads, dim, batch, width = 8, 17, 2, 32, 5, 3
    tables = torch.from_numpy(gen.permutation(blocks)[:batch * width].astype(np.int64)).view(batch, width)
    tables[3, 1] = -1          # request 3 appends into an unallocated page -> skipped
    offsets = torch.tensor([0, 7, 9, 12, 23], dtype=torch.int64)
    offsets[4] = 3 * block_size  # past the table -> skipped
    return {"key_cache": randn(gen, (blocks, block_size, kv_heads, dim), dtype),
            "value_cache": randn(gen, (blocks, block_size, kv_heads, dim), dtype),
            "block_tables": tables, "token_offsets": offsets,
            "key": randn(gen, (batch, kv_heads, dim), dtype),
            "value": randn(gen, (batch, kv_heads, dim), dtype), "block_size": block_size}


# --------------------------------------------------------------------------- prefill

def ragged_small(dtype=torch.float32, dim=16, seed=631):
    """Packed prefill of tests/test_ragged_kernels.py:17-24 (bs 4, offsets [0,3,8])."""
    gen = rng(seed)
    key = randn(gen, (8, 4, 2, dim), dtype)
    value = randn(gen, (8, 4, 2, dim), dtype)
    q = randn(gen, (8, 4, dim), dtype)
    meta = [torch.tensor(x, dtype=torch.int64) for x in
            ([0, 3, 8], [5, 1], [[5, 1, -1], [2, 7, -1]], [8, 6])]
    return {"q": q, "key_cache": key, "value_cache": value, "cu_seqlens_q": meta[0],
            "query_starts": meta[1], "block_tables": meta[2], "context_lens": meta[3],
            "block_size": 4}


def config4(seed=105, requests=16, chunk=128, block_size=16, shared_tokens=512,
            sharers=8, cow_request=3, cow_start=496, heads=HQ, kv_heads=HKV, head_dim=D,
            dtype=torch.bfloat16):
    """Ragged chunked prefill with a shared prefix and one copy-on-write page.

    Requests ``0..sharers-1`` attach the same ``shared_tokens // block_size``
    pages (prefix >= ``shared_tokens``); request ``cow_request`` starts its chunk
    at ``cow_start``, inside the last shared page, so that page must be copied
    to a private page before the chunk's K/V are scattered.  Other prefixes are
    U[0, 1024] rounded down to the block size.  Returns the pre-CoW tables,
    the CoW pair and the post-CoW tables.
    """
    gen = rng(seed)
    prefixes = [int(x) // block_size * block_size for x in gen.integers(0, 1025, size=requests)]
    shared_pages = shared_tokens // block_size
    for r in range(sharers):
        prefixes[r] = max(prefixes[r], shared_tokens)
    prefixes[cow_request] = cow_start
    pages_needed = [(p + chunk + block_size - 1) // block_size for p in prefixes]
    private = sum(n - (shared_pages if r < sharers else 0) for r, n in enumerate(pages_needed))
    pool_blocks = shared_pages + private + 1 + 8       # +1 CoW target, +8 spare
    perm = gen.permutation(pool_blocks).astype(np.int64).tolist()
    shared = perm[:shared_pages]
    cursor = shared_pages
    tables = []
    for r, n in enumerate(pages_needed):
        own = n - (shared_pages if r < sharers else 0)
        table = (list(shared) if r < sharers else []) + perm[cursor:cursor + own]
        cursor += own
        tables.append(table)
    cow_target = perm[cursor]
    cow_index = cow_start // block_size
    cow_pair = (tables[cow_request][cow_index], cow_target)
    cow_tables = [list(t) for t in tables]
    cow_tables[cow_request][cow_index] = cow_target
    key_cache = randn(gen, (pool_blocks, block_size, kv_heads, head_dim), dtype)
    value_cache = randn(gen, (pool_blocks, block_size, kv_heads, head_dim), dtype)
    total = requests * chunk
    q = randn(gen, (total, heads, head_dim), dtype)
    key = randn(gen, (total, kv_heads, head_dim), dtype)
    value = randn(gen, (total, kv_heads, head_dim), dtype)
    tokens = [[int(t) for t in gen.integers(0, 151936, size=chunk)] for _ in range(requests)]
    return {"q": q, "key": key, "value": value, "key_cache": key_cache, "value_cache": value_cache,
            "tables": tables, "cow_tables": cow_tables, "cow_pair": cow_pair, "starts": prefixes,
            "tokens": tokens, "block_size": block_size, "num_blocks": pool_blocks}


def ragged_prefill_case(dtype, *, head_dim=D, heads=HQ, kv_heads=HKV, block_size=16,
                        starts=(0, 37, 130, 5), chunks=(70, 1, 129, 33), seed=106, spare=5):
    """Generic packed prefill case: K/V for every context position already in the pages."""
    gen = rng(seed)
    lengths = [s + c for s, c in zip(starts, chunks)]
    pages = [(n + block_size - 1) // block_size for n in lengths]
    width = max(pages)
    blocks = sum(pages) + spare
    perm = gen.permutation(blocks).astype(np.int64)
    table = np.full((len(starts), width), -1, dtype=np.int64)
    cursor = 0
    for r, n in enumerate(pages):
        table[r, :n] = perm[cursor:cursor + n]
        cursor += n
    offsets = np.concatenate([[0], np.cumsum(chunks)]).astype(np.int64)
    key = randn(gen, (blocks, block_size, kv_heads, head_dim), dtype)
    value = randn(gen, (blocks, block_size, kv_heads, head_dim), dtype)
    q = randn(gen, (int(offsets[-1]), heads, head_dim), dtype)
    return {"q": q, "key_cache": key, "value_cache": value,
            "cu_seqlens_q": torch.from_numpy(offsets), "query_starts": torch.tensor(starts, dtype=torch.int64),
            "block_tables": torch.from_numpy(table), "context_lens": torch.tensor(lengths, dtype=torch.int64),
            "block_size": block_size}


# --------------------------------------------------------------------------- metadata

METADATA_GOLDEN = {  # tests/test_ragged_model.py:42-53, literal values
    "args": ([[5, 6, 7], [8, 9]], [[3, 1, -1], [3, 2]], [4, 4]),
    "block_size": 4, "num_blocks": 16,
    "expected": {"input_ids": [5, 6, 7, 8, 9], "positions": [4, 5, 6, 4, 5],
                 "slot_mapping": [4, 5, 6, 8, 9], "cu_seqlens_q": [0, 3, 5],
                 "context_lens": [7, 6]},
}

METADATA_REJECTIONS = [  # tests/test_ragged_model.py:56-73 (tensor-typed cases omitted)
    ([[]], [[0]], [0], "nonempty"),
    ([[1]], [[0]], [-1], "nonnegative"),
    ([[1]], [[0]], [True], "integers"),
    ([[1]], [[0]], [], "equal batch"),
    ([[-1]], [[0]], [0], "nonnegative"),
    ([[1]], [[16]], [0], "out of range"),
    ([[1]], [[0, 0]], [0], "duplicate physical"),
    ([[1]], [[0, -1, 2]], [0], "trailing"),
    ([[1, 2]], [[0]], [3], "capacity"),
    ([[1], [2]], [[0], [0]], [0, 0], "duplicate writable"),
    ([[1], [2]], [[0], [0]], [0, 1], "shared by requests"),
    ([[1 << 64]], [[0]], [0], "int64"),
]


def metadata_random(seed=107, requests=24, block_size=16, max_start=700, max_chunk=90):
    """A larger ragged batch: random starts/chunks, private pages from a permutation."""
    gen = rng(seed)
    starts = [int(x) for x in gen.integers(0, max_start, size=requests)]
    chunks = [int(x) for x in gen.integers(1, max_chunk, size=requests)]
    pages = [(s + c + block_size - 1) // block_size + int(gen.integers(0, 3)) for s, c in zip(starts, chunks)]
    blocks = sum(pages) + 11
    perm = gen.permutation(blocks).astype(np.int64).tolist()
    tables, cursor = [], 0
    for n in pages:
        tables.append(perm[cursor:cursor + n])
        cursor += n
    tokens = [[int(t) for t in gen.integers(0, 151936, size=c)] for c in chunks]
    return {"tokens": tokens, "tables": tables, "starts": starts, "block_size": block_size,
            "num_blocks": blocks}


# ------------------------------------------------------------------- decode step

def qwen3_weights(config, dtype, *, seed, std=0.02, device="cpu"):
    """Seeded Qwen3 weights in the fused layouts of enable_projection_fusion.

    Projections and the embedding ~ N(0, std) (numpy PCG64, drawn in the order
    embed, then per layer q|k|v, o, gate|up, down), norms = 1.  Returns a
    namespace with the attributes the decode step and the oracle read.
    """
    from types import SimpleNamespace

    gen = rng(seed)
    cfg = config

    def normal(*shape):
        return (randn(gen, shape, torch.float32) * std).to(dtype).to(device)

    def ones(n):
        return torch.ones(n, dtype=dtype, device=device)

    h, d, i = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    embed = normal(cfg.vocab_size, h)
    layers = []
    for _ in range(cfg.num_hidden_layers):
        qkv = normal((cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * d, h)
        o = normal(h, cfg.num_attention_heads * d)
        gate_up, down = normal(2 * i, h), normal(h, i)
        layers.append(SimpleNamespace(input_norm=ones(h), qkv=qkv, q_norm=ones(d), k_norm=ones(d), o=o,
                                      post_norm=ones(h), gate_up=gate_up, down=down))
    return SimpleNamespace(embed=embed, norm=ones(h), layers=layers, lm_head=embed)


def qwen3_tiny_config():
    """A small architecture of the Qwen3 family for CPU golden runs of the reference model."""
    from types import SimpleNamespace

    return SimpleNamespace(vocab_size=128, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=8, rms_norm_eps=1e-6,
                           rope_theta=1000000.0, max_position_embeddings=4096, tie_word_embeddings=True)


def qwen3_decode_case(config, dtype, *, contexts, block_size, seed, pool_slack=1.25):
    """One batched decode step: random N(0,1) KV history of ``contexts[b]`` tokens, token ids U[0, vocab).

    Request b appends at position ``contexts[b]``; its pages are a slice of a
    seeded permutation of the pool.  Pools are ``[layers, blocks, block_size,
    kv_heads, head_dim]``.
    """
    gen = rng(seed)
    pages = [(c + 1 + block_size - 1) // block_size for c in contexts]
    width = max(pages)
    blocks = math.ceil(pool_slack * sum(pages))
    perm = gen.permutation(blocks).astype(np.int64)
    table = np.full((len(contexts), width), -1, dtype=np.int64)
    used = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[used:used + n]
        used += n
    shape = (config.num_hidden_layers, blocks, block_size, config.num_key_value_heads, config.head_dim)
    key_pool, value_pool = randn(gen, shape, dtype), randn(gen, shape, dtype)
    ids = torch.from_numpy(gen.integers(0, config.vocab_size, size=len(contexts)).astype(np.int64))
    return {"input_ids": ids, "positions": torch.tensor(contexts, dtype=torch.int64),
            "block_tables": torch.from_numpy(table), "key_pool": key_pool, "value_pool": value_pool,
            "block_size": block_size}
