"""The Qwen3 decode step over an FP8 KV pool (``FP8KVCachePool``).

Checker: the same step over a bf16 pool that holds the FP8 pool's history
dequantised (exact: the scale is a power of two and every FP8 value fits
bf16).  The two steps then differ only by the quantisation of the newest
token's K/V in each layer, which the FP8 step stores and attends to in FP8.

Bars:
  * logits within the decode-step tolerance of tests/test_gpu_decode_step.py
    (atol=0.25, rtol=0.01);
  * layer 0's appended rows bit-exact with the oracle's quantisation of the
    bf16 step's appended rows (both steps compute them with the same kernels
    from the same inputs);
  * nothing else in the FP8 pools changed;
  * the step captured in a CUDA graph replays to the eager step's logits.
"""

import numpy as np
import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.cache import FP8KVCachePool
from myvllm_mini_engine_b200.engine.qwen3 import Qwen3DecodeStep
from oracle import fp8_kv
from test_gpu_decode_step import ATOL, RTOL, appended, model_case

pytestmark = pytest.mark.gpu
SCALE = 1.0 / 32  # power of two: the dequantised history is exact in bf16


def fp8_copy(cfg, pool, fmt):
    """An FP8 pool holding ``pool``'s history quantised; ``pool`` is overwritten with its dequantised values."""
    shape = pool.shape
    fp8 = FP8KVCachePool(shape.num_layers, shape.num_blocks, shape.block_size, shape.num_kv_heads, shape.head_dim,
                         k_scale=SCALE, v_scale=SCALE, kv_format=fmt)
    slots = torch.arange(shape.num_blocks * shape.block_size, device="cuda")
    rows = (-1, shape.num_kv_heads, shape.head_dim)
    for layer in range(shape.num_layers):
        fp8.write_slots(layer, slots, pool.key[layer].view(rows), pool.value[layer].view(rows), validate=False)
    view = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    pool.key.copy_((fp8.key.view(view).float() * SCALE).to(pool.key.dtype))
    pool.value.copy_((fp8.value.view(view).float() * SCALE).to(pool.value.dtype))
    return fp8


@pytest.mark.parametrize("fused,fmt", [(True, "e4m3"), (False, "e5m2"), (True, "e5m2")],
                         ids=["fused-e4m3", "cublas-e5m2", "fused-e5m2"])
def test_fp8_pool_step_matches_the_bf16_step_on_the_dequantised_pool(cuda_device, fused, fmt):
    contexts = (1, 17, 255, 256, 700, 1031) + tuple(int(x) for x in cases.rng(43).integers(1, 2048, 30))
    if fused:
        contexts = contexts[:Qwen3DecodeStep.FUSED_MAX_BATCH]
    cfg, weights, pool, tables, ids, positions = model_case(contexts, seed=41)
    fp8 = fp8_copy(cfg, pool, fmt)
    step16 = Qwen3DecodeStep(cfg, weights, pool, fused_projections=fused)
    step8 = Qwen3DecodeStep(cfg, weights, fp8, fused_projections=fused)
    before = (fp8.key.clone(), fp8.value.clone())
    logits8 = step8.forward_decode_batch(ids, tables, positions)
    logits16 = step16.forward_decode_batch(ids, tables, positions)
    torch.testing.assert_close(logits8.float(), logits16.float(), atol=ATOL, rtol=RTOL)
    bs = pool.shape.block_size
    for mine, theirs, old in ((fp8.key, pool.key, before[0]), (fp8.value, pool.value, before[1])):
        pages, offsets, rows16 = appended(theirs, tables, positions, bs)
        codes = fp8_kv.quantize(rows16[0].cpu(), SCALE, fmt)
        assert np.array_equal(mine[0, pages, offsets].cpu().numpy(), codes)
        rest = mine.clone()
        rest[:, pages, offsets] = old[:, pages, offsets]
        assert torch.equal(rest, old)
    assert _lib.device_status() == 0


def test_fp8_pool_step_replays_in_a_cuda_graph(cuda_device):
    contexts = (5, 64, 300, 999)
    cfg, weights, pool, tables, ids, positions = model_case(contexts, seed=47, layers=4)
    fp8 = fp8_copy(cfg, pool, "e4m3")
    step = Qwen3DecodeStep(cfg, weights, fp8)
    start = (fp8.key.clone(), fp8.value.clone())
    eager = step.forward_decode_batch(ids, tables, positions)
    fp8.key.copy_(start[0])
    fp8.value.copy_(start[1])
    capture = torch.cuda.Stream()
    capture.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(capture):
        step.forward_decode_batch(ids, tables, positions)  # warm-up: workspaces exist before capture
    capture.synchronize()
    fp8.key.copy_(start[0])
    fp8.value.copy_(start[1])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=capture):
        out = step.forward_decode_batch(ids, tables, positions)
    fp8.key.copy_(start[0])
    fp8.value.copy_(start[1])
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert _lib.device_status() == 0
