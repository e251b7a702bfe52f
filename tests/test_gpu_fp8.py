"""FP8 (E4M3 / E5M2) KV pool on the GPU against the CPU oracle (oracle/fp8_kv.py).

The quantising scatter must match the oracle byte for byte.  Decode attention
over an FP8 pool is compared with the fp32 oracle run on the dequantised pool
(``code * scale``), at the decode tolerances: fp16 atol=rtol=2e-3, bf16
atol=rtol=1e-2.
"""

import numpy as np
import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.kernels import paged_attention, paged_attention_fp8, write_kv_cache_slots_fp8
from oracle import fp8_kv

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
K_SCALE, V_SCALE = 0.0125, 0.0095  # N(0,1) data spans about +-400 codes' worth of range


def fp8_pools(c, k_scale=K_SCALE, v_scale=V_SCALE, fmt="e4m3"):
    """The case's 16-bit pools quantised by the oracle (uint8, CPU)."""
    k = torch.from_numpy(fp8_kv.quantize(c["key_cache"], k_scale, fmt))
    v = torch.from_numpy(fp8_kv.quantize(c["value_cache"], v_scale, fmt))
    return k, v


def run_both(c, dtype, k_scale=K_SCALE, v_scale=V_SCALE, validate=True, tables=None, lens=None, fmt="e4m3"):
    kq, vq = fp8_pools(c, k_scale, v_scale, fmt)
    tables = c["block_tables"] if tables is None else tables
    lens = c["context_lens"] if lens is None else lens
    expected = fp8_kv.paged_attention_fp8_fp32(c["query"], kq, vq, tables, lens, c["block_size"], k_scale, v_scale,
                                               fmt)
    actual = paged_attention_fp8(c["query"].cuda(), kq.cuda(), vq.cuda(), tables.cuda(), lens.cuda(),
                                 c["block_size"], k_scale, v_scale, kv_format=fmt, validate=validate)
    return actual, expected


def assert_close(actual, expected_fp32, dtype):
    tol = TOL[dtype]
    torch.testing.assert_close(actual.float().cpu(), expected_fp32, atol=tol, rtol=tol)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("src", [torch.float32, torch.float16, torch.bfloat16])
def test_quantising_scatter_is_bit_exact(cuda_device, src, fmt):
    gen = np.random.default_rng(5)
    blocks, bs, hkv, dim, tokens = 12, 16, 4, 64, 150
    mags = gen.choice([1e-6, 1e-3, 0.05, 1.0, 3.0, 6.0], size=(2, tokens + 8, hkv, dim))
    data = torch.from_numpy((gen.standard_normal((2, tokens + 8, hkv, dim)) * mags).astype(np.float32)).to(src)
    # edge values: saturation (+-inf and beyond 448*scale), signed zero, ties, the subnormal range
    edge = torch.tensor([float("inf"), -float("inf"), -0.0, 0.0, 1e9, -1e9, 448 * K_SCALE, 2 ** -10 * K_SCALE,
                         -(2 ** -10) * K_SCALE, 2 ** -9 * K_SCALE, 1.0625 * K_SCALE, 1.1875 * K_SCALE],
                        dtype=torch.float32).to(src)
    data[0, 0, 0, :edge.numel()] = edge
    data[1, 2, 1, :edge.numel()] = edge / K_SCALE * V_SCALE
    # token-strided views (every other token of a larger buffer)
    key, value = data[0, ::2], data[1, ::2]
    n = key.shape[0]
    slots = torch.from_numpy(gen.permutation(blocks * bs)[:n].astype(np.int64))
    slots[3] = -1
    slots[7] = blocks * bs + 5  # outside the capacity: skipped
    init = torch.from_numpy(gen.integers(0, 256, size=(2, blocks, bs, hkv, dim), dtype=np.uint8))
    kc, vc = init[0].clone(), init[1].clone()
    fp8_kv.scatter_slots_fp8(kc, vc, slots, key.contiguous(), value.contiguous(), K_SCALE, V_SCALE, fmt)
    gk, gv = init[0].cuda(), init[1].cuda()
    write_kv_cache_slots_fp8(gk, gv, slots.cuda(), key.cuda(), value.cuda(), K_SCALE, V_SCALE, kv_format=fmt,
                             validate=False)
    torch.cuda.synchronize()
    assert torch.equal(gk.cpu(), kc) and torch.equal(gv.cpu(), vc)
    # the float8 dtype view reads back the same values the oracle decodes
    view = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    got = gk.view(view).float().cpu().numpy()
    want = fp8_kv.decode_fp8(kc.numpy(), fmt)
    assert np.array_equal(np.isnan(got), np.isnan(want)) and np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dim", [32, 64, 96, 128, 192, 256])
def test_decode_matches_oracle_on_dequantised_pool(cuda_device, dtype, dim, fmt):
    c = cases.decode_case(dtype, head_dim=dim)
    actual, expected = run_both(c, dtype, fmt=fmt)
    assert actual.dtype == dtype and actual.shape == c["query"].shape
    assert_close(actual, expected, dtype)


@pytest.mark.parametrize("block_size,lengths,heads,kv_heads", [
    (16, (256, 255), 8, 1), (32, (257, 1025, 9), 16, 8), (16, (4097,), 16, 8), (256, (513, 1, 300), 16, 8),
    (1, (7, 33), 16, 8), (24, (100, 47), 32, 4), (16, (65,), 16, 16), (16, (700, 3000), 32, 2),
])
def test_block_partition_and_group_boundaries(cuda_device, block_size, lengths, heads, kv_heads):
    c = cases.decode_case(torch.bfloat16, block_size=block_size, lengths=lengths, heads=heads, kv_heads=kv_heads)
    for fmt in ("e4m3", "e5m2"):
        actual, expected = run_both(c, torch.bfloat16, fmt=fmt)
        assert_close(actual, expected, torch.bfloat16)


def test_scales_apply_and_equal_the_16bit_decode_of_the_dequantised_pool(cuda_device):
    c = cases.decode_case(torch.float16, lengths=(33, 600, 129))
    for k_scale, v_scale in ((K_SCALE, V_SCALE), (0.5, 2.0), (1.0, 1.0)):
        kq, vq = fp8_pools(c, k_scale, v_scale)
        fp8 = paged_attention_fp8(c["query"].cuda(), kq.cuda(), vq.cuda(), c["block_tables"].cuda(),
                                  c["context_lens"].cuda(), 16, k_scale, v_scale)
        # the 16-bit decode of the dequantised pool (rounded to fp16; exact for power-of-two scales)
        kd = fp8_kv.dequantize(kq, k_scale).to(torch.float16).cuda()
        vd = fp8_kv.dequantize(vq, v_scale).to(torch.float16).cuda()
        ref = paged_attention(c["query"].cuda(), kd, vd, c["block_tables"].cuda(), c["context_lens"].cuda(), 16)
        assert_close(fp8, ref.float().cpu(), torch.float16)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_trusted_mode_invalid_pages_and_lengths(cuda_device, fmt):
    c = cases.decode_case(torch.bfloat16, lengths=(65, 300, 17))
    tables = c["block_tables"].clone()
    tables[0].fill_(-1)
    tables[1, 3] = 1 << 40
    lens = c["context_lens"].clone()
    lens[2] = 10_000
    actual, expected = run_both(c, torch.bfloat16, validate=False, tables=tables, lens=lens, fmt=fmt)
    assert torch.isfinite(actual).all() and not actual[0].any() and not actual[2].any()
    assert_close(actual, expected, torch.bfloat16)
    assert _lib.device_status() == 0


def test_rejects_unsupported_arguments(cuda_device):
    c = cases.decode_case(torch.bfloat16, head_dim=80, lengths=(5,))
    kq, vq = fp8_pools(c)
    args = [c["query"].cuda(), kq.cuda(), vq.cuda(), c["block_tables"].cuda(), c["context_lens"].cuda(), 16]
    with pytest.raises(RuntimeError, match="head_dim"):
        paged_attention_fp8(*args, K_SCALE, V_SCALE)
    c = cases.decode_case(torch.float32, head_dim=64, lengths=(5,))
    kq, vq = fp8_pools(c)
    with pytest.raises(RuntimeError, match="FP16/BF16"):
        paged_attention_fp8(c["query"].cuda(), kq.cuda(), vq.cuda(), c["block_tables"].cuda(),
                            c["context_lens"].cuda(), 16, K_SCALE, V_SCALE)
    with pytest.raises(ValueError, match="kv_format"):
        paged_attention_fp8(c["query"].cuda().half(), kq.cuda(), vq.cuda(), c["block_tables"].cuda(),
                            c["context_lens"].cuda(), 16, K_SCALE, V_SCALE, kv_format="e3m4")
    with pytest.raises(ValueError, match="finite and positive"):
        paged_attention_fp8(c["query"].cuda().half(), kq.cuda(), vq.cuda(), c["block_tables"].cuda(),
                            c["context_lens"].cuda(), 16, 0.0, V_SCALE)


@pytest.mark.parametrize("dtype,fmt", [(torch.float16, "e4m3"), (torch.bfloat16, "e5m2")])
def test_scatter_then_decode_replays_in_a_cuda_graph(cuda_device, dtype, fmt):
    """One captured step: quantise the new tokens into the pool, then decode; replays see new inputs."""
    c = cases.decode_case(dtype, lengths=(40, 255, 517, 3))
    kq, vq = fp8_pools(c, fmt=fmt)
    gk, gv = kq.cuda(), vq.cuda()
    tables, lens = c["block_tables"].cuda(), c["context_lens"].cuda()
    batch, _, dim = c["query"].shape
    hkv = c["key_cache"].shape[2]
    gen = torch.Generator().manual_seed(3)
    new_k = torch.randn(batch, hkv, dim, generator=gen).to(dtype).cuda()
    new_v = torch.randn(batch, hkv, dim, generator=gen).to(dtype).cuda()
    # slot of each request's last token
    last = (lens - 1).cpu()
    slots = torch.tensor([int(c["block_tables"][b, int(last[b]) // 16]) * 16 + int(last[b]) % 16
                          for b in range(batch)], dtype=torch.int64).cuda()
    query = c["query"].cuda()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        paged_attention_fp8(query, gk, gv, tables, lens, 16, K_SCALE, V_SCALE, kv_format=fmt, validate=False)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        write_kv_cache_slots_fp8(gk, gv, slots, new_k, new_v, K_SCALE, V_SCALE, kv_format=fmt, validate=False)
        out = paged_attention_fp8(query, gk, gv, tables, lens, 16, K_SCALE, V_SCALE, kv_format=fmt, validate=False)
    for step in range(2):
        new_k.normal_()
        new_v.normal_()
        query.mul_(0.9)
        graph.replay()
        torch.cuda.synchronize()
        kc, vc = kq.clone(), vq.clone()
        fp8_kv.scatter_slots_fp8(kc, vc, slots.cpu(), new_k.cpu(), new_v.cpu(), K_SCALE, V_SCALE, fmt)
        assert torch.equal(gk.cpu(), kc) and torch.equal(gv.cpu(), vc)
        expected = fp8_kv.paged_attention_fp8_fp32(query.cpu(), kc, vc, c["block_tables"], c["context_lens"], 16,
                                                   K_SCALE, V_SCALE, fmt)
        assert_close(out, expected, dtype)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("block_size", [16, 32])
def test_runs_across_contiguous_pages(cuda_device, block_size):
    """Pages laid out back to back: one staged copy spans several pages (and whole tiles)."""
    c = cases.decode_case(torch.bfloat16, block_size=block_size, lengths=(1000, 37, 513))
    width = c["block_tables"].shape[1]
    c["block_tables"] = torch.arange(3 * width, dtype=torch.int64).view(3, width)
    actual, expected = run_both(c, torch.bfloat16)
    assert_close(actual, expected, torch.bfloat16)
    # mixed: contiguous pages with a few holes (-1 pages are masked in trusted mode)
    tables = c["block_tables"].clone()
    tables[0, 5] = -1
    tables[2, 1] = -1
    actual, expected = run_both(c, torch.bfloat16, validate=False, tables=tables)
    assert_close(actual, expected, torch.bfloat16)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_pool_range_write_attend_gather_and_copy_on_write(cuda_device, fmt):
    from myvllm_mini_engine_b200.cache import FP8KVCachePool

    gen = torch.Generator().manual_seed(17)
    layers, blocks, bs, hkv, dim = 2, 24, 16, 4, 64
    pool = FP8KVCachePool(layers, blocks, bs, hkv, dim, k_scale=K_SCALE, v_scale=V_SCALE, kv_format=fmt)
    ids, offset, tokens = [5, 17, 2, 9], 3, 50
    key = torch.randn(tokens, hkv, dim, generator=gen).to(torch.bfloat16)
    value = torch.randn(tokens, hkv, dim, generator=gen).to(torch.bfloat16)
    pool.write_range(1, ids, offset, key.cuda(), value.cuda())
    positions = torch.arange(tokens) + offset
    slots = torch.tensor(ids)[positions // bs] * bs + positions % bs
    kc = torch.zeros(blocks, bs, hkv, dim, dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    fp8_kv.scatter_slots_fp8(kc, vc, slots, key, value, K_SCALE, V_SCALE, fmt)
    assert torch.equal(pool.key[1].cpu(), kc) and torch.equal(pool.value[1].cpu(), vc)
    assert not pool.key[0].any() and not pool.value[0].any()
    k_rows, v_rows = pool.dequantized(1, ids, offset + tokens)
    assert torch.equal(k_rows[offset:].cpu(), fp8_kv.dequantize(kc.view(-1, hkv, dim)[slots], K_SCALE, fmt))
    assert torch.equal(v_rows[offset:].cpu(), fp8_kv.dequantize(vc.view(-1, hkv, dim)[slots], V_SCALE, fmt))
    query = torch.randn(2, 8, dim, generator=gen).to(torch.bfloat16)
    tables = torch.tensor([ids, ids], dtype=torch.int64)
    lens = torch.tensor([offset + tokens, 20], dtype=torch.int64)
    out = pool.attend(1, query.cuda(), tables.cuda(), lens.cuda())
    expected = fp8_kv.paged_attention_fp8_fp32(query, kc, vc, tables, lens, bs, K_SCALE, V_SCALE, fmt)
    assert_close(out, expected, torch.bfloat16)
    pool.copy_blocks([(17, 20)])
    torch.cuda.synchronize()
    assert torch.equal(pool.key[:, 20], pool.key[:, 17]) and torch.equal(pool.value[:, 20], pool.value[:, 17])


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_ragged_prefill_over_fp8_pool_matches_oracle(cuda_device, fmt):
    """BASELINE config 4's ragged batch (16 x 128-token chunks over prefixes up to 1024) on an FP8 pool."""
    from myvllm_mini_engine_b200.engine import PrefillBatch
    from myvllm_mini_engine_b200.kernels import paged_prefill_attention_fp8
    from oracle import prefill as prefill_oracle

    c = cases.config4()
    bs = c["block_size"]
    batch = PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"], block_size=bs,
                                        num_blocks=c["num_blocks"], device="cuda")
    kq = torch.from_numpy(fp8_kv.quantize(c["key_cache"], K_SCALE, fmt))
    vq = torch.from_numpy(fp8_kv.quantize(c["value_cache"], V_SCALE, fmt))
    meta = (batch.cu_seqlens_q, batch.query_starts, batch.block_tables, batch.context_lens)
    out = paged_prefill_attention_fp8(c["q"].cuda(), kq.cuda(), vq.cuda(), *meta, bs, K_SCALE, V_SCALE,
                                      kv_format=fmt)
    expected = prefill_oracle.paged_prefill_fp32(c["q"].float(), fp8_kv.dequantize(kq, K_SCALE, fmt),
                                                 fp8_kv.dequantize(vq, V_SCALE, fmt), *(t.cpu() for t in meta), bs)
    assert out.dtype == c["q"].dtype and out.shape == c["q"].shape
    assert_close(out, expected, c["q"].dtype)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_ragged_prefill_over_fp8_pool_in_several_chunks(cuda_device, dtype):
    """More packed tokens than one launch chunk of the CUDA-core route (4096 query rows): the chunk
    loop (ticket reset per chunk, q/out offsets, a shorter last chunk) over a small-head model
    (head_dim 96, which the tensor-core route does not take), fp16 and bf16 queries, both formats."""
    from myvllm_mini_engine_b200.engine import PrefillBatch
    from myvllm_mini_engine_b200.kernels import paged_prefill_attention_fp8
    from oracle import prefill as prefill_oracle

    gen = np.random.default_rng(61)
    bs, heads, kv_heads, dim = 16, 2, 1, 96
    starts = [0, 48, 3, 200]
    chunks = [2500, 1800, 700, 1333]  # 6333 packed tokens: two chunks of the route
    pages = [(s + n + bs - 1) // bs for s, n in zip(starts, chunks)]
    blocks = sum(pages) + 3
    perm = gen.permutation(blocks).tolist()
    tables, at = [], 0
    for n in pages:
        tables.append(perm[at:at + n])
        at += n
    tokens = [gen.integers(0, 1000, size=n).tolist() for n in chunks]
    batch = PrefillBatch.from_sequences(tokens, tables, starts, block_size=bs, num_blocks=blocks, device="cuda")
    q = torch.from_numpy(gen.standard_normal((sum(chunks), heads, dim), dtype=np.float32)).to(dtype)
    cache = torch.from_numpy(gen.standard_normal((2, blocks, bs, kv_heads, dim), dtype=np.float32))
    meta = (batch.cu_seqlens_q, batch.query_starts, batch.block_tables, batch.context_lens)
    for fmt in ("e4m3", "e5m2"):
        kq = torch.from_numpy(fp8_kv.quantize(cache[0], K_SCALE, fmt))
        vq = torch.from_numpy(fp8_kv.quantize(cache[1], V_SCALE, fmt))
        out = paged_prefill_attention_fp8(q.cuda(), kq.cuda(), vq.cuda(), *meta, bs, K_SCALE, V_SCALE, kv_format=fmt)
        expected = prefill_oracle.paged_prefill_fp32(q.float(), fp8_kv.dequantize(kq, K_SCALE, fmt),
                                                     fp8_kv.dequantize(vq, V_SCALE, fmt), *(t.cpu() for t in meta),
                                                     bs)
        assert out.dtype == dtype and out.shape == q.shape
        assert_close(out, expected, dtype)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype,fmt,dim,heads,kv_heads,bs", [
    (torch.float16, "e4m3", 64, 8, 2, 16),     # dense copy
    (torch.bfloat16, "e4m3", 64, 4, 1, 8),     # dense copy
    (torch.bfloat16, "e5m2", 128, 16, 16, 32),  # codes converted in the kernel, bf16 Q converted too
    (torch.float16, "e4m3", 128, 8, 1, 8),      # in the kernel, fp16 Q, 8-row page boxes
    (torch.bfloat16, "e4m3", 128, 32, 2, 256),  # in the kernel, 128-row page boxes
])
def test_ragged_prefill_over_fp8_pool_tensor_core_route(cuda_device, dtype, fmt, dim, heads, kv_heads, bs):
    """Both tensor-core routes (head_dim 128: codes staged and converted inside the kernel; 64:
    a dense 16-bit copy first): ragged chunks over prefixes, a request with no prefix,
    a one-token chunk, a shared prefix page, table entries past the context holding garbage page
    ids (never converted, masked), and an exact repeat (the copy is rebuilt each call)."""
    from myvllm_mini_engine_b200.engine import PrefillBatch
    from myvllm_mini_engine_b200.kernels import paged_prefill_attention_fp8
    from oracle import prefill as prefill_oracle

    gen = np.random.default_rng(dim + heads + bs)
    starts = [0, 2 * bs + 37, 2 * bs, 5]  # requests 1 and 2 share their first (prefix) page
    chunks = [150, 61, 1, 200]
    pages = [(s + n + bs - 1) // bs for s, n in zip(starts, chunks)]
    blocks = sum(pages) + 4
    perm = gen.permutation(blocks).tolist()
    tables, at = [], 0
    for n in pages:
        tables.append(perm[at:at + n])
        at += n
    tables[2][0] = tables[1][0]  # shared prefix page
    tokens = [gen.integers(0, 1000, size=n).tolist() for n in chunks]
    batch = PrefillBatch.from_sequences(tokens, tables, starts, block_size=bs, num_blocks=blocks, device="cuda")
    bt = batch.block_tables.clone()
    lens = batch.context_lens.cpu().tolist()
    for b in range(bt.shape[0]):  # entries past the context: out-of-range and in-range ids alike
        used = (lens[b] + bs - 1) // bs
        for j in range(used, bt.shape[1]):
            bt[b, j] = blocks + 7 if (j % 2) else perm[j % blocks]
    q = torch.from_numpy(gen.standard_normal((sum(chunks), heads, dim), dtype=np.float32)).to(dtype)
    cache = torch.from_numpy(gen.standard_normal((2, blocks, bs, kv_heads, dim), dtype=np.float32))
    kq = torch.from_numpy(fp8_kv.quantize(cache[0], K_SCALE, fmt))
    vq = torch.from_numpy(fp8_kv.quantize(cache[1], V_SCALE, fmt))
    meta = (batch.cu_seqlens_q, batch.query_starts, bt, batch.context_lens)
    expected = prefill_oracle.paged_prefill_fp32(q.float(), fp8_kv.dequantize(kq, K_SCALE, fmt),
                                                 fp8_kv.dequantize(vq, V_SCALE, fmt), *(t.cpu() for t in meta), bs)
    first = None
    for _ in range(2):
        out = paged_prefill_attention_fp8(q.cuda(), kq.cuda(), vq.cuda(), *meta, bs, K_SCALE, V_SCALE,
                                          kv_format=fmt, validate=False)
        assert out.dtype == dtype and out.shape == q.shape
        assert_close(out, expected, dtype)
        if first is None:
            first = out.clone()
        else:
            assert torch.equal(out, first)
    assert _lib.device_status() == 0


def test_fp8_prefill_workspace_follows_the_route(cuda_device):
    """Config 4's shape: head_dim 128 stages the codes inside the tcgen05 kernel (no workspace);
    head_dim 64 needs the dense 16-bit copy of every table entry's page (two pools + table);
    head_dim 96 takes the CUDA-core route (token map + decode workspace)."""
    lib = _lib.load()
    code = _lib.dtype_code(torch.bfloat16)
    tokens, requests, hq, hkv, blocks, bs, width = 2048, 16, 16, 8, 455, 16, 71
    query = lambda dim: lib.minikv_paged_prefill_fp8_workspace_bytes(tokens, requests, hq, hkv, dim, blocks, bs,
                                                                      width, 128, code)
    assert query(128) == 0
    assert query(64) >= 2 * requests * width * bs * hkv * 64 * 2 + requests * width * 8
    assert query(96) > 0
