"""Ragged paged prefill on the GPU against the CPU oracle, including BASELINE config 4
(copy-on-write of a shared prefix page + slot scatter + prefill)."""

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from myvllm_mini_engine_b200.engine import PrefillBatch
from myvllm_mini_engine_b200.kernels import copy_blocks, paged_prefill_attention, write_kv_cache_slots
from oracle import kv_write, metadata, prefill

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1e-2}
PREFILL = np.load(Path(__file__).resolve().parent / "golden" / "golden_prefill.npz")
NAMES = ("q", "key_cache", "value_cache", "cu_seqlens_q", "query_starts", "block_tables", "context_lens")


def assert_close(actual, expected_fp32, dtype):
    torch.testing.assert_close(actual.float().cpu(), expected_fp32, atol=TOL[dtype], rtol=TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dim", [16, 128])
def test_small_packed_prefill_on_nondefault_stream(cuda_device, dtype, dim):
    c = cases.ragged_small(dtype, dim)
    expected = prefill.per_token_fp32(*[c[k] for k in NAMES], 4)
    args = [c[k].cuda() for k in NAMES]
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        result = paged_prefill_attention(*args, 4)
    torch.cuda.current_stream().wait_stream(stream)
    assert_close(result, expected, dtype)
    if dtype == torch.float32 and dim == 16:
        golden = torch.from_numpy(PREFILL["small/out"]).view(torch.float32).reshape(result.shape)
        assert_close(result, golden, dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dim,heads,kv_heads", [(128, 16, 8), (64, 8, 8), (128, 32, 4), (96, 16, 8), (256, 16, 8)])
def test_ragged_prefill_matches_oracle(cuda_device, dtype, dim, heads, kv_heads):
    c = cases.ragged_prefill_case(dtype, head_dim=dim, heads=heads, kv_heads=kv_heads)
    expected = prefill.paged_prefill_fp32(*[c[k] for k in NAMES], c["block_size"])
    result = paged_prefill_attention(*[c[k].cuda() for k in NAMES], c["block_size"])
    assert_close(result, expected, dtype)


@pytest.mark.parametrize("name", ["fp16", "bf16"])
def test_ragged_prefill_matches_reference_golden(cuda_device, name):
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16}[name]
    c = cases.ragged_prefill_case(dtype)
    result = paged_prefill_attention(*[c[k].cuda() for k in NAMES], c["block_size"])
    golden = torch.from_numpy(PREFILL[f"ragged_{name}/out"]).view(dtype).reshape(result.shape)
    assert_close(result, golden.float(), dtype)


def test_context_beyond_dense_prefill_limit(cuda_device):
    block, context = 32, 8193
    gen = cases.rng(77)
    pages = (context + block - 1) // block
    key = cases.randn(gen, (pages, block, 1, 16), torch.float16)
    value = cases.randn(gen, (pages, block, 1, 16), torch.float16)
    q = cases.randn(gen, (1, 2, 16), torch.float16)
    tables = torch.from_numpy(gen.permutation(pages).astype(np.int64)).view(1, -1)
    meta = [torch.tensor([0, 1]), torch.tensor([context - 1]), tables, torch.tensor([context])]
    expected = prefill.per_token_fp32(q, key, value, meta[0], meta[1], meta[2], meta[3], block)
    actual = paged_prefill_attention(q.cuda(), key.cuda(), value.cuda(), meta[0].cuda(), meta[1].cuda(),
                                     meta[2].cuda(), meta[3].cuda(), block)
    assert_close(actual, expected, torch.float16)


def test_empty_packed_queries(cuda_device):
    c = cases.ragged_small(torch.bfloat16, 16)
    empty = torch.empty(0, dtype=torch.int64, device="cuda")
    result = paged_prefill_attention(c["q"][:0].cuda(), c["key_cache"].cuda(), c["value_cache"].cuda(),
                                     torch.tensor([0], device="cuda"), empty,
                                     torch.empty(0, 0, dtype=torch.int64, device="cuda"), empty, 4)
    assert result.shape == (0, 4, 16)


def test_config4_copy_on_write_scatter_and_prefill(cuda_device):
    c = cases.config4()
    bs = c["block_size"]
    # oracle path (CPU): CoW copy, metadata, scatter, prefill
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.copy_blocks(kc.unsqueeze(0), vc.unsqueeze(0), [c["cow_pair"]])
    meta = metadata.prefill_metadata(c["tokens"], c["cow_tables"], c["starts"], block_size=bs,
                                     num_blocks=c["num_blocks"])
    t = {k: torch.tensor(v, dtype=torch.int64) for k, v in meta.items()}
    kv_write.write_kv_cache_slots(kc, vc, t["slot_mapping"], c["key"], c["value"])
    expected = prefill.paged_prefill_fp32(c["q"], kc, vc, t["cu_seqlens_q"], t["query_starts"],
                                          t["block_tables"], t["context_lens"], bs)
    # GPU path: device CoW, device metadata, scatter, tcgen05 prefill
    gk, gv = c["key_cache"].cuda(), c["value_cache"].cuda()
    copy_blocks(gk.unsqueeze(0), gv.unsqueeze(0), [c["cow_pair"]])
    batch = PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"], block_size=bs,
                                        num_blocks=c["num_blocks"], device="cuda")
    for name, values in meta.items():
        assert getattr(batch, name).tolist() == values, name
    write_kv_cache_slots(gk, gv, batch.slot_mapping, c["key"].cuda(), c["value"].cuda(), validate=False)
    assert torch.equal(gk.cpu(), kc) and torch.equal(gv.cpu(), vc)
    out = paged_prefill_attention(c["q"].cuda(), gk, gv, batch.cu_seqlens_q, batch.query_starts,
                                  batch.block_tables, batch.context_lens, bs, validate=False)
    assert_close(out, expected, torch.bfloat16)
    rows = torch.from_numpy(PREFILL["config4/rows"])
    golden = torch.from_numpy(PREFILL["config4/out_rows"]).view(torch.bfloat16).reshape(-1, 16, 128)
    assert_close(out[rows.cuda()], golden.float(), torch.bfloat16)


def _kernel_names(fn):
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {evt.name for evt in prof.events() if evt.device_type == torch.autograd.DeviceType.CUDA}


@pytest.mark.parametrize("dtype,dim,heads,kv_heads,expect_tc", [
    (torch.bfloat16, 128, 16, 8, True), (torch.float16, 64, 8, 8, True), (torch.bfloat16, 128, 32, 4, True),
    (torch.bfloat16, 96, 16, 8, False), (torch.float32, 128, 16, 8, False),
])
def test_tensor_core_route_selection(cuda_device, dtype, dim, heads, kv_heads, expect_tc):
    c = cases.ragged_prefill_case(dtype, head_dim=dim, heads=heads, kv_heads=kv_heads)
    args = [c[k].cuda() for k in NAMES]
    paged_prefill_attention(*args, c["block_size"])  # load + warm up
    names = _kernel_names(lambda: paged_prefill_attention(*args, c["block_size"]))
    used_tc = any("paged_prefill_tc_kernel" in n for n in names)
    assert used_tc == expect_tc, names
    if not expect_tc:
        assert any("paged_decode_kernel" in n for n in names), names


def sub_batch(args, r):
    """Request r of a packed prefill batch as a batch of its own (same caches)."""
    q, kc, vc, cu, starts, tables, lens = args
    lo, hi = int(cu[r]), int(cu[r + 1])
    return (q[lo:hi].contiguous(), kc, vc, torch.tensor([0, hi - lo], dtype=torch.int64, device=q.device),
            starts[r:r + 1].contiguous(), tables[r:r + 1].contiguous(), lens[r:r + 1].contiguous())


@pytest.mark.parametrize("dtype,dim", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_prefill_output_of_a_request_does_not_depend_on_the_batch(cuda_device, dtype, dim):
    # Tensor-core route: every (query tile, kv head) item of a request is computed by
    # one CTA over the request's own keys in a fixed order (query tiles never mix
    # requests), so the rows of a request alone and inside a batch are bit-identical.
    # (The CUDA-core route runs the split-KV decode over the batch's tokens, whose
    # split points depend on the whole batch: equal within tolerance, not in bits.)
    c = cases.ragged_prefill_case(dtype, head_dim=dim)
    args = [c[k].cuda() for k in NAMES]
    batched = paged_prefill_attention(*args, c["block_size"])
    cu = c["cu_seqlens_q"]
    for r in range(len(cu) - 1):
        alone = paged_prefill_attention(*sub_batch(args, r), c["block_size"])
        assert torch.equal(alone, batched[int(cu[r]):int(cu[r + 1])]), f"request {r}"


@pytest.mark.parametrize("dtype,dim", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_prefill_replays_in_a_cuda_graph(cuda_device, dtype, dim):
    # The ragged prefill is captured once with static metadata and query buffers;
    # replays with new contents of the same shapes match eager calls on them.
    c = cases.ragged_prefill_case(dtype, head_dim=dim)
    static = [c[k].cuda() for k in NAMES]
    bs = c["block_size"]
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        paged_prefill_attention(*static, bs, validate=False)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        out = paged_prefill_attention(*static, bs, validate=False)
    q, _, _, cu, starts, tables, lens = static
    gen = torch.Generator(device="cuda").manual_seed(5)
    for step in range(2):
        # new queries and a shifted split of the same token count between the requests
        q.copy_(torch.randn(q.shape, device="cuda", generator=gen).to(dtype))
        counts = (cu[1:] - cu[:-1]).tolist()
        if step == 1:
            counts[0], counts[2] = counts[0] - 20, counts[2] + 20
        new_cu = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int64, device="cuda")
        new_starts = starts.clone()
        new_starts[2] = max(0, int(starts[2]) - 20)  # request 2 keeps within its pages
        cu.copy_(new_cu)
        starts.copy_(new_starts)
        lens.copy_(starts + (cu[1:] - cu[:-1]))
        graph.replay()
        expected = paged_prefill_attention(*static, bs)
        torch.cuda.synchronize()
        assert torch.equal(out, expected), f"replay {step}"
