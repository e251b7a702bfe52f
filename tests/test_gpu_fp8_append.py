"""Fused KV append + decode over FP8 pools (``paged_attention_fp8_with_append``).

The two-call path it replaces is ``write_kv_cache_slots_fp8`` of the new rows
at each request's slot for ``token_offsets[b]``, then ``paged_attention_fp8``
over ``token_offsets + 1`` tokens.  The fused launch must leave the pools
byte-identical to the oracle (the 16-bit append of data.py:67-81 followed by the
quantisation of oracle/fp8_kv.py) and to the two calls, and return the two
calls' output bit for bit (same plan, same staged bytes); against the fp32
oracle over the dequantised pools it stays within the decode tolerances (fp16
atol=rtol=2e-3, bf16 atol=rtol=1e-2).
"""

import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.kernels import (paged_attention_fp8, paged_attention_fp8_with_append,
                                             write_kv_cache_slots_fp8)
from oracle import fp8_kv, kv_write

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
K_SCALE, V_SCALE = 0.0125, 0.0095


def quantized(c, fmt):
    """The case's pools quantised by the oracle (uint8, CPU)."""
    return (torch.from_numpy(fp8_kv.quantize(c["key_cache"], K_SCALE, fmt)),
            torch.from_numpy(fp8_kv.quantize(c["value_cache"], V_SCALE, fmt)))


def slots_of(c):
    """Pool slot of each request's new token, -1 where the offset or its page is out of range."""
    tables, offsets, bs = c["block_tables"], c["token_offsets"], c["block_size"]
    pages = c["key_cache"].shape[0]
    out = []
    for b, off in enumerate(offsets.tolist()):
        page = tables[b, off // bs].item() if 0 <= off < tables.shape[1] * bs else -1
        out.append(page * bs + off % bs if 0 <= page < pages else -1)
    return torch.tensor(out, dtype=torch.int64)


def fused(c, kq, vq, fmt, **kw):
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    kc, vc = kq.cuda(), vq.cuda()
    out = paged_attention_fp8_with_append(g["query"], kc, vc, g["block_tables"], g["token_offsets"], g["key"],
                                          g["value"], c["block_size"], K_SCALE, V_SCALE, kv_format=fmt, **kw)
    return out, kc, vc


def two_calls(c, kq, vq, fmt):
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    kc, vc = kq.cuda(), vq.cuda()
    write_kv_cache_slots_fp8(kc, vc, slots_of(c).cuda(), g["key"], g["value"], K_SCALE, V_SCALE, kv_format=fmt,
                             validate=False)
    out = paged_attention_fp8(g["query"], kc, vc, g["block_tables"], g["token_offsets"] + 1, c["block_size"],
                              K_SCALE, V_SCALE, kv_format=fmt, validate=False)
    return out, kc, vc


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("dtype,dim,heads,kv_heads,block_size", [
    (torch.bfloat16, 128, 16, 8, 16),    # the Qwen3 shape
    (torch.float16, 64, 128, 1, 32),     # a group of 128 query heads: several CTAs per kv head
    (torch.bfloat16, 256, 16, 8, 16),    # kv-head groups of CTAs, each quantises its heads of the row
    (torch.float16, 32, 8, 2, 8),
])
def test_fp8_fused_append_matches_oracle_and_two_calls(cuda_device, fmt, dtype, dim, heads, kv_heads, block_size):
    contexts = [0, 15, 16, 300, 1023]
    c = cases.append_decode_case(dtype, batch=len(contexts), contexts=contexts, block_size=block_size, seed=91,
                                 heads=heads, kv_heads=kv_heads, head_dim=dim)
    kq, vq = quantized(c, fmt)
    actual, kc, vc = fused(c, kq, vq, fmt)
    # oracle: the 16-bit append, then the pools quantised element by element
    k16, v16 = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(k16, v16, c["block_tables"], c["token_offsets"], c["key"], c["value"],
                                  block_size)
    ko = torch.from_numpy(fp8_kv.quantize(k16, K_SCALE, fmt))
    vo = torch.from_numpy(fp8_kv.quantize(v16, V_SCALE, fmt))
    assert torch.equal(kc.cpu(), ko) and torch.equal(vc.cpu(), vo)
    expected = fp8_kv.paged_attention_fp8_fp32(c["query"], ko, vo, c["block_tables"], c["context_lens"],
                                               block_size, K_SCALE, V_SCALE, fmt)
    tol = TOL[dtype]
    torch.testing.assert_close(actual.float().cpu(), expected, atol=tol, rtol=tol)
    separate, kc2, vc2 = two_calls(c, kq, vq, fmt)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(actual, separate)
    assert _lib.device_status() == 0


def test_fp8_fused_append_keeps_the_guards_of_the_two_calls(cuda_device):
    c = cases.append_decode_case(torch.bfloat16, batch=5, contexts=[40, 7, 100, 63, 5], block_size=16, seed=92)
    tables = c["block_tables"].clone()
    offsets = c["token_offsets"].clone()
    offsets[1] = -3                           # negative offset: no write, zero row
    offsets[2] = tables.shape[1] * 16         # beyond the table: no write, zero row
    tables[3, 63 // 16] = c["key_cache"].shape[0] + 5  # the new token's page is invalid: no write, token masked
    c = dict(c, block_tables=tables, token_offsets=offsets)
    kq, vq = quantized(c, "e4m3")
    actual, kc, vc = fused(c, kq, vq, "e4m3", validate=False)
    separate, kc2, vc2 = two_calls(c, kq, vq, "e4m3")
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert not actual[1].any() and not actual[2].any()
    assert torch.equal(actual, separate)
    with pytest.raises(RuntimeError, match="offset out of range"):
        fused(c, kq, vq, "e4m3", validate=True)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_chained_fp8_fused_append_replays_in_a_graph(cuda_device, fmt):
    """The new rows come from the previous kernel (a scale of the inputs) and the offsets predate it."""
    dtype = torch.bfloat16
    c = cases.append_decode_case(dtype, batch=6, contexts=[3, 99, 512, 17, 64, 250], block_size=16, seed=93)
    kq, vq = quantized(c, fmt)
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    kc, vc = kq.cuda(), vq.cuda()
    base_k, base_v = g["key"].clone(), g["value"].clone()

    def step():
        g["key"].copy_(base_k * 2)   # the producing kernel of the new rows
        g["value"].copy_(base_v * 2)
        return paged_attention_fp8_with_append(g["query"], kc, vc, g["block_tables"], g["token_offsets"], g["key"],
                                               g["value"], 16, K_SCALE, V_SCALE, kv_format=fmt, validate=False,
                                               chained=True)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        eager = step().clone()
    side.synchronize()
    after = kc.clone(), vc.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        out = step()
    kc.copy_(kq)
    vc.copy_(vq)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert torch.equal(kc, after[0]) and torch.equal(vc, after[1])
    c2 = dict(c, key=(c["key"].float() * 2).to(dtype), value=(c["value"].float() * 2).to(dtype))
    separate, kc2, vc2 = two_calls(c2, kq, vq, fmt)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(out, separate)
    del graph
    assert _lib.device_status() == 0
