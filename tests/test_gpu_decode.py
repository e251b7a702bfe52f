"""Paged decode attention on the GPU against the CPU oracle.

Tolerances (stated by the north star): fp16 atol=rtol=2e-3, bf16 atol=rtol=1e-2
against the fp32 oracle; fp32 is held to 1e-4.  Shapes follow the reference's
own CUDA tests (tests/test_cuda_paged_attention.py) and BASELINE configs 1-3.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.kernels import paged_attention, write_kv_cache_batch
from oracle import kv_write, paged_decode

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1e-2}
DECODE = np.load(Path(__file__).resolve().parent / "golden" / "golden_decode.npz")


def args_of(c, device="cuda"):
    names = ("query", "key_cache", "value_cache", "block_tables", "context_lens")
    return [c[k].to(device) for k in names]


def assert_close(actual, expected_fp32, dtype):
    tol = TOL[dtype]
    torch.testing.assert_close(actual.float().cpu(), expected_fp32, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dim", [16, 32, 64, 80, 96, 128, 192, 256])
def test_gqa_split_kv_matches_oracle(cuda_device, dtype, dim):
    c = cases.decode_case(dtype, head_dim=dim)
    expected = paged_decode.paged_attention_fp32(*args_of(c, "cpu"), c["block_size"])
    actual = paged_attention(*args_of(c), c["block_size"])
    assert actual.dtype == dtype and actual.shape == c["query"].shape
    assert_close(actual, expected, dtype)


@pytest.mark.parametrize("block_size,lengths,heads,kv_heads", [
    (4, (1,), 4, 4), (16, (256, 255), 8, 1), (32, (257, 1025, 9), 16, 8), (16, (4097,), 16, 8),
    (256, (513, 1, 300), 16, 8), (1, (7, 33), 16, 8), (24, (100, 47), 32, 4), (16, (65,), 16, 16),
])
def test_block_and_partition_boundaries(cuda_device, block_size, lengths, heads, kv_heads):
    c = cases.decode_case(torch.bfloat16, block_size=block_size, lengths=lengths, heads=heads, kv_heads=kv_heads)
    expected = paged_decode.paged_attention_fp32(*args_of(c, "cpu"), block_size)
    actual = paged_attention(*args_of(c), block_size)
    assert_close(actual, expected, torch.bfloat16)


@pytest.mark.parametrize("name", ["sweep_bf16_d128", "sweep_fp16_d80", "sweep_fp32_d16"])
def test_matches_reference_golden_outputs(cuda_device, name):
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[name.split("_")[1]]
    dim = int(name.split("_d")[1])
    c = cases.decode_case(dtype, head_dim=dim, lengths=(17, 57, 130))
    golden = torch.from_numpy(DECODE[name + "/out"]).view(dtype).reshape(c["query"].shape)
    actual = paged_attention(*args_of(c), c["block_size"])
    # golden is the reference torch path rounded to `dtype`: allow one output rounding step
    assert_close(actual, golden.float(), dtype)


@pytest.mark.parametrize("name", ["config1", "config2", "config3"])
def test_baseline_config_append_then_decode(cuda_device, name):
    c = getattr(cases, name)()
    dtype = c["query"].dtype
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(kc, vc, c["block_tables"], c["token_offsets"], c["key"], c["value"],
                                  c["block_size"])
    expected = paged_decode.paged_attention_fp32(c["query"], kc, vc, c["block_tables"], c["context_lens"],
                                                 c["block_size"])
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                         g["value"], g["block_size"], validate=False)
    actual = paged_attention(g["query"], g["key_cache"], g["value_cache"], g["block_tables"], g["context_lens"],
                             g["block_size"], validate=False)
    assert_close(actual, expected, dtype)
    golden = torch.from_numpy(DECODE[name + "/out"]).view(dtype).reshape(actual.shape)
    assert_close(actual, golden.float(), dtype)


def test_headline_shape_matches_oracle_on_sampled_requests(cuda_device):
    c = cases.headline_case()
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                         g["value"], g["block_size"], validate=False)
    actual = paged_attention(g["query"], g["key_cache"], g["value_cache"], g["block_tables"], g["context_lens"],
                             16, validate=False).cpu()
    kc, vc = g["key_cache"].cpu(), g["value_cache"].cpu()
    rows = [0, 7, 19, 31]
    expected = paged_decode.paged_attention_fp32(c["query"][rows], kc, vc, c["block_tables"][rows],
                                                 c["context_lens"][rows], 16)
    assert_close(actual[rows], expected, torch.bfloat16)
    # size-independent property: a permutation of the batch permutes the output rows
    perm = torch.randperm(32, generator=torch.Generator().manual_seed(5))
    shuffled = paged_attention(g["query"][perm.cuda()].contiguous(), g["key_cache"], g["value_cache"],
                               g["block_tables"][perm.cuda()].contiguous(), g["context_lens"][perm.cuda()].contiguous(),
                               16, validate=False).cpu()
    torch.testing.assert_close(shuffled, actual[perm], atol=1e-2, rtol=1e-2)


def test_rejects_bad_metadata_and_noncontiguous_query(cuda_device):
    args = args_of(cases.decode_case(torch.float16))
    args[4][0] = 0
    with pytest.raises(RuntimeError, match="context length"):
        paged_attention(*args, 16)
    args[4][0] = 17
    args[3][0, 0] = -1
    with pytest.raises(RuntimeError, match="physical block"):
        paged_attention(*args, 16)
    args[3][0, 0] = 0
    args[0] = args[0].transpose(0, 1).contiguous().transpose(0, 1)
    with pytest.raises(RuntimeError, match="contiguous"):
        paged_attention(*args, 16)


def test_current_stream_and_trusted_invalid_indices_give_zero_rows(cuda_device):
    c = cases.decode_case(torch.bfloat16, lengths=(65, 300, 17))
    args = args_of(c)
    expected = paged_decode.paged_attention_fp32(*args_of(c, "cpu"), 16)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        actual = paged_attention(*args, 16, validate=False)
    torch.cuda.current_stream().wait_stream(stream)
    assert_close(actual, expected, torch.bfloat16)
    # corrupt pages and lengths: never read out of bounds; rows become zero (reference trusted mode)
    tables = args[3].clone()
    tables[0].fill_(-1)
    tables[1, 3] = 1 << 40
    lens = args[4].clone()
    lens[2] = 10_000
    out = paged_attention(args[0], args[1], args[2], tables, lens, 16, validate=False)
    oracle = paged_decode.paged_attention_trusted_fp32(args[0].cpu(), args[1].cpu(), args[2].cpu(), tables.cpu(),
                                                       lens.cpu(), 16)
    assert torch.isfinite(out).all() and not out[0].any() and not out[2].any()
    assert_close(out, oracle, torch.bfloat16)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("block_size", [16, 32, 256])
def test_graph_replay_with_new_lengths_and_queries(cuda_device, dtype, block_size):
    c = cases.decode_case(dtype, block_size=block_size, lengths=(1, 255, 257, 519))
    args = args_of(c)
    original_k, original_v = args[1].clone(), args[2].clone()
    paged_attention(*args, block_size, validate=False)  # warm-up (loads the library)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = paged_attention(*args, block_size, validate=False)
    args[4].copy_(torch.tensor([256, 128, 16, 1], device="cuda"))
    args[0].mul_(0.75)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.current_stream().wait_stream(stream)
    expected = paged_decode.paged_attention_fp32(*[a.cpu() for a in args], block_size)
    assert_close(captured, expected, dtype)
    assert torch.equal(original_k, args[1]) and torch.equal(original_v, args[2])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_chained_decode_after_append_in_a_graph(cuda_device, dtype):
    """Append + chained decode (prologue overlapped with the append) equals the plain launches, bit for bit."""
    c = cases.append_decode_case(dtype, batch=6, contexts=[0, 15, 16, 300, 1023, 77], block_size=16, seed=91)
    names = ("key_cache", "value_cache", "block_tables", "token_offsets", "key", "value")
    g = {k: c[k].cuda() for k in names + ("query", "context_lens")}
    plain_k, plain_v = g["key_cache"].clone(), g["value_cache"].clone()
    write_kv_cache_batch(plain_k, plain_v, g["block_tables"], g["token_offsets"], g["key"], g["value"], 16,
                         validate=False)
    expected = paged_attention(g["query"], plain_k, plain_v, g["block_tables"], g["context_lens"], 16,
                               validate=False)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        paged_attention(g["query"], g["key_cache"], g["value_cache"], g["block_tables"], g["context_lens"], 16,
                        validate=False, chained=True)  # workspace of this stream, outside the graph
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                             g["value"], 16, validate=False)
        out = paged_attention(g["query"], g["key_cache"], g["value_cache"], g["block_tables"], g["context_lens"],
                              16, validate=False, chained=True)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, expected)
    assert torch.equal(g["key_cache"], plain_k) and torch.equal(g["value_cache"], plain_v)
    assert _lib.device_status() == 0
