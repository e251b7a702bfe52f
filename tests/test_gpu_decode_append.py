"""Fused KV append + paged decode (``paged_attention_with_append``) against the two-call path.

The reference runs ``write_kv_cache_batch`` and then ``paged_attention`` over
``positions + 1`` (mini_engine/model/native_qwen3.py:188-196).  The fused
operator must leave the pools bit-identical to the oracle's append (restating
data.py:67-81) and return attention within the decode tolerances of the fp32
oracle over the appended pools; invalid offsets and pages follow the guards of
the two CUDA calls (no write, zero rows).
"""

import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.kernels import paged_attention, paged_attention_with_append, write_kv_cache_batch
from oracle import kv_write, paged_decode

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1e-2}


def gpu(c):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}


def fused(g, **kw):
    return paged_attention_with_append(g["query"], g["key_cache"], g["value_cache"], g["block_tables"],
                                       g["token_offsets"], g["key"], g["value"], g["block_size"], **kw)


def check_against_oracle(c, actual, g):
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(kc, vc, c["block_tables"], c["token_offsets"], c["key"], c["value"],
                                  c["block_size"])
    assert torch.equal(g["key_cache"].cpu(), kc) and torch.equal(g["value_cache"].cpu(), vc)
    expected = paged_decode.paged_attention_fp32(c["query"], kc, vc, c["block_tables"], c["context_lens"],
                                                 c["block_size"])
    tol = TOL[c["query"].dtype]
    torch.testing.assert_close(actual.float().cpu(), expected, atol=tol, rtol=tol)


@pytest.mark.parametrize("name", ["config1", "config2", "config3"])
def test_fused_append_decode_matches_oracle_and_two_calls(cuda_device, name):
    c = getattr(cases, name)()
    g, two = gpu(c), gpu(c)
    actual = fused(g)
    check_against_oracle(c, actual, g)
    write_kv_cache_batch(two["key_cache"], two["value_cache"], two["block_tables"], two["token_offsets"],
                         two["key"], two["value"], two["block_size"], validate=False)
    separate = paged_attention(two["query"], two["key_cache"], two["value_cache"], two["block_tables"],
                               two["context_lens"], two["block_size"], validate=False)
    assert torch.equal(g["key_cache"], two["key_cache"]) and torch.equal(g["value_cache"], two["value_cache"])
    tol = TOL[c["query"].dtype]
    torch.testing.assert_close(actual.float(), separate.float(), atol=tol, rtol=tol)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype,dim,heads,kv_heads,block_size", [
    (torch.bfloat16, 256, 16, 8, 16),    # two kv-head groups of CTAs, each writes its heads of the row
    (torch.float16, 64, 128, 1, 32),     # a group of 128 query heads: several CTAs per kv head
    (torch.float16, 128, 8, 8, 1),       # MHA, one token per page
    (torch.float32, 80, 16, 4, 64),      # CUDA-core consumer
])
def test_fused_append_decode_shapes(cuda_device, dtype, dim, heads, kv_heads, block_size):
    contexts = [0, 15, 16, 300, 1023]
    c = cases.append_decode_case(dtype, batch=len(contexts), contexts=contexts, block_size=block_size, seed=77,
                                 heads=heads, kv_heads=kv_heads, head_dim=dim)
    g = gpu(c)
    actual = fused(g, validate=True)
    check_against_oracle(c, actual, g)
    assert _lib.device_status() == 0


def test_fused_append_keeps_the_guards_of_the_two_calls(cuda_device):
    c = cases.append_decode_case(torch.bfloat16, batch=5, contexts=[40, 7, 100, 63, 5], block_size=16, seed=78)
    tables = c["block_tables"].clone()
    offsets = c["token_offsets"].clone()
    offsets[1] = -3                           # negative offset: no write, zero row
    offsets[2] = tables.shape[1] * 16         # beyond the table: no write, zero row
    tables[3, 63 // 16] = c["key_cache"].shape[0] + 5  # the new token's page is invalid: no write, token masked
    c = dict(c, block_tables=tables, token_offsets=offsets)
    g, two = gpu(c), gpu(c)
    actual = fused(g, validate=False)
    write_kv_cache_batch(two["key_cache"], two["value_cache"], two["block_tables"], two["token_offsets"],
                         two["key"], two["value"], 16, validate=False)
    separate = paged_attention(two["query"], two["key_cache"], two["value_cache"], two["block_tables"],
                               two["token_offsets"] + 1, 16, validate=False)
    assert torch.equal(g["key_cache"], two["key_cache"]) and torch.equal(g["value_cache"], two["value_cache"])
    assert not actual[1].any() and not actual[2].any()
    torch.testing.assert_close(actual.float(), separate.float(), atol=1e-2, rtol=1e-2)
    with pytest.raises(RuntimeError, match="offset out of range"):
        fused(g, validate=True)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_chained_fused_append_replays_in_a_graph(cuda_device, dtype):
    """The new rows come from the previous kernel (a scale of the inputs) and the offsets predate it."""
    c = cases.append_decode_case(dtype, batch=6, contexts=[3, 99, 512, 17, 64, 250], block_size=16, seed=79)
    g = gpu(c)
    base_k, base_v = g["key"].clone(), g["value"].clone()
    pools = g["key_cache"].clone(), g["value_cache"].clone()

    def step():
        g["key"].copy_(base_k * 2)   # the producing kernel of the new rows
        g["value"].copy_(base_v * 2)
        return fused(g, validate=False, chained=True)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        eager = step().clone()
    side.synchronize()
    after = g["key_cache"].clone(), g["value_cache"].clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        out = step()
    g["key_cache"].copy_(pools[0])
    g["value_cache"].copy_(pools[1])
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert torch.equal(g["key_cache"], after[0]) and torch.equal(g["value_cache"], after[1])
    c2 = dict(c, key=(c["key"].float() * 2).to(dtype), value=(c["value"].float() * 2).to(dtype))
    check_against_oracle(c2, out, g)
    del graph
    assert _lib.device_status() == 0
