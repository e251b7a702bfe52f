"""KV scatter / append / range write / copy-on-write on the GPU: bit-exact against the oracle."""

import pytest
import torch

import cases
from myvllm_mini_engine_b200.kernels import (copy_blocks, write_kv_cache, write_kv_cache_batch,
                                             write_kv_cache_slots)
from oracle import kv_write

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def cuda(c):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dim", [16, 128])
def test_slot_scatter_bit_exact_on_nondefault_stream_with_strided_sources(cuda_device, dtype, dim):
    c = cases.slots_case(dtype, dim)
    expected_k, expected_v = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_slots(expected_k, expected_v, c["slot_mapping"], c["key"], c["value"])
    g = cuda(c)
    packed = torch.cat([c["key"], c["value"]], dim=1).cuda()
    key, value = packed[:, :2], packed[:, 2:]  # split-projection views: token-strided, rows contiguous
    assert not key.is_contiguous()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        write_kv_cache_slots(g["key_cache"], g["value_cache"], g["slot_mapping"], key, value)
    torch.cuda.current_stream().wait_stream(stream)
    assert torch.equal(g["key_cache"].cpu(), expected_k) and torch.equal(g["value_cache"].cpu(), expected_v)


def test_slot_scatter_trusted_mode_skips_out_of_range_slots(cuda_device):
    c = cases.slots_case(torch.bfloat16, 128)
    slots = torch.tensor([5, -1, 7, 32, 10, 11, 28, 1 << 40])
    expected_k, expected_v = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_slots(expected_k, expected_v, slots, c["key"], c["value"])
    g = cuda(c)
    write_kv_cache_slots(g["key_cache"], g["value_cache"], slots.cuda(), g["key"], g["value"], validate=False)
    assert torch.equal(g["key_cache"].cpu(), expected_k) and torch.equal(g["value_cache"].cpu(), expected_v)


def test_empty_scatter_is_a_noop(cuda_device):
    c = cuda(cases.slots_case(torch.float16, 16))
    before = c["key_cache"].clone()
    empty = torch.empty(0, dtype=torch.int64, device="cuda")
    write_kv_cache_slots(c["key_cache"], c["value_cache"], empty, c["key"][:0], c["value"][:0])
    assert torch.equal(c["key_cache"], before)


@pytest.mark.parametrize("dtype", DTYPES)
def test_range_write_crosses_pages_bit_exact(cuda_device, dtype):
    c = cases.range_case(dtype)
    expected_k, expected_v = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache(expected_k, expected_v, c["block_ids"], c["token_offset"], c["key"], c["value"],
                            c["block_size"])
    g = cuda(c)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        write_kv_cache(g["key_cache"], g["value_cache"], g["block_ids"], g["token_offset"], g["key"], g["value"],
                       g["block_size"])
    torch.cuda.current_stream().wait_stream(stream)
    assert torch.equal(g["key_cache"].cpu(), expected_k) and torch.equal(g["value_cache"].cpu(), expected_v)


def test_range_write_validate_rejects_bad_page(cuda_device):
    g = cuda(cases.range_case())
    with pytest.raises(RuntimeError, match="physical block id"):
        write_kv_cache(g["key_cache"], g["value_cache"], torch.tensor([4, 9, 5], device="cuda"), 1,
                       g["key"], g["value"], 4)


@pytest.mark.parametrize("dtype", DTYPES)
def test_batch_append_bit_exact_and_skips_invalid_rows(cuda_device, dtype):
    c = cases.batch_write_case(dtype)
    expected_k, expected_v = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(expected_k, expected_v, c["block_tables"], c["token_offsets"], c["key"],
                                  c["value"], c["block_size"])
    g = cuda(c)
    write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                         g["value"], g["block_size"], validate=False)
    assert torch.equal(g["key_cache"].cpu(), expected_k) and torch.equal(g["value_cache"].cpu(), expected_v)
    with pytest.raises(RuntimeError, match="offset out of range"):
        write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                             g["value"], g["block_size"], validate=True)


@pytest.mark.parametrize("name", ["config1", "config2", "config3"])
def test_config_appends_bit_exact(cuda_device, name):
    c = getattr(cases, name)()
    expected_k, expected_v = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(expected_k, expected_v, c["block_tables"], c["token_offsets"], c["key"],
                                  c["value"], c["block_size"])
    g = cuda(c)
    write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                         g["value"], g["block_size"], validate=False)
    assert torch.equal(g["key_cache"].cpu(), expected_k) and torch.equal(g["value_cache"].cpu(), expected_v)


@pytest.mark.parametrize("dtype", DTYPES)
def test_copy_blocks_bit_exact_over_all_layers(cuda_device, dtype):
    gen = cases.rng(71)
    pool_k = cases.randn(gen, (3, 20, 16, 8, 128), dtype)
    pool_v = cases.randn(gen, (3, 20, 16, 8, 128), dtype)
    pairs = [(3, 17), (4, 9), (19, 0)]
    expected_k, expected_v = pool_k.clone(), pool_v.clone()
    kv_write.copy_blocks(expected_k, expected_v, pairs)
    gk, gv = pool_k.cuda(), pool_v.cuda()
    copy_blocks(gk, gv, pairs)
    assert torch.equal(gk.cpu(), expected_k) and torch.equal(gv.cpu(), expected_v)
    with pytest.raises(ValueError, match="distinct"):
        copy_blocks(gk, gv, [(1, 2), (2, 3)])


def test_copy_blocks_and_scatter_capture_in_cuda_graph(cuda_device):
    gen = cases.rng(72)
    pool_k = cases.randn(gen, (2, 12, 16, 8, 128), torch.bfloat16).cuda()
    pool_v = cases.randn(gen, (2, 12, 16, 8, 128), torch.bfloat16).cuda()
    pairs = torch.tensor([[1, 5]], device="cuda")
    slots = torch.tensor([5 * 16 + 3, 5 * 16 + 4], device="cuda")
    k = cases.randn(gen, (2, 8, 128), torch.bfloat16).cuda()
    v = cases.randn(gen, (2, 8, 128), torch.bfloat16).cuda()
    expected_k, expected_v = pool_k.cpu(), pool_v.cpu()
    kv_write.copy_blocks(expected_k, expected_v, [(1, 5)])
    kv_write.write_kv_cache_slots(expected_k[1], expected_v[1], slots.cpu(), k.cpu(), v.cpu())
    graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        copy_blocks(pool_k, pool_v, pairs, validate=False)
        write_kv_cache_slots(pool_k[1], pool_v[1], slots, k, v, validate=False)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(pool_k.cpu(), expected_k) and torch.equal(pool_v.cpu(), expected_v)
