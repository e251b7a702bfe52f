"""The drop-in inside the reference engine, on the GPU.

``integration.install`` rebinds the reference package's CUDA backends to this
package; these tests then run the reference's own model, CUDA-graph bucket
and batch runtime, unchanged, and compare them with the same reference code on
its torch backends, on the same GPU and weights:

* ``NativeQwen3`` prefill + decode (``model/native_qwen3.py``), as the
  reference's own check does (tests/test_cuda_paged_attention.py:104-124:
  tiny Qwen3 config, torch vs cuda decode, logits close and argmax equal);
* ``DecodeGraphBucket.capture`` / ``replay_metadata`` (engine/cuda_graph.py:196-275)
  with the rebound decode, KV append and metadata ops inside the graph;
* ``NativeBatchRuntime`` prefill + decode steps with a prefix-cache hit
  (engine/runtime.py:187-299): the same greedy tokens as the torch runtime.

Embedding lookup and RoPE are outside the hot path; with ``data_backend="cuda"``
the reference would JIT-build its own extension for them, so they run the
reference's torch implementation here (``_torch_side_ops``).  Needs the
reference copy under baseline/_ref (skipped without it).
"""

import pytest
import torch

from myvllm_mini_engine_b200 import _lib, integration

pytestmark = pytest.mark.gpu

CONFIG = dict(vocab_size=71, hidden_size=32, intermediate_size=64, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, max_position_embeddings=128)


def _torch_side_ops(nq):
    """Route the model's embedding and RoPE calls to the reference's torch implementations."""
    from mini_engine.kernels import data as ref_data

    rope, embed = ref_data.apply_rope, ref_data.embedding_lookup

    def apply_rope(q, k, cos, sin, *, backend="torch", validate=True):
        if cos.ndim == 2:  # the cuda layout passes [tokens, D/2]; the torch one [tokens, 1, D/2]
            cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        return rope(q, k, cos, sin, backend="torch")

    def embedding_lookup(weight, input_ids, *, backend="torch", validate=True):
        return embed(weight, input_ids, backend="torch")

    nq.apply_rope_backend = apply_rope
    nq.embedding_lookup = embedding_lookup


def _models(reference_engine, dtype, seed=8):
    """(reference model on torch backends, the same weights on the installed CUDA backends)."""
    import mini_engine.model.native_qwen3 as nq
    from mini_engine.model import NativeQwen3, Qwen3Config

    patched = integration.install(reference_engine)
    assert any(name.endswith("native_qwen3.paged_attention") for name in patched)
    _torch_side_ops(nq)
    cfg = Qwen3Config(**CONFIG)
    torch.manual_seed(seed)
    ref = NativeQwen3(cfg, "math", "torch", "torch", "torch").to(device="cuda", dtype=dtype).eval()
    new = NativeQwen3(cfg, "cuda", "cuda", "torch", "cuda").to(device="cuda", dtype=dtype).eval()
    new.load_state_dict(ref.state_dict())
    return ref, new


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_reference_model_prefill_and_decode_on_installed_ops(cuda_device, reference_engine, dtype):
    ref, new = _models(reference_engine, dtype)
    ref_cache, new_cache = ref.create_cache(8, 4), new.create_cache(8, 4)
    ids = torch.tensor([1, 5, 6, 8, 7], device="cuda")
    blocks = [6, 1, 4, 0]
    a = ref(ids, ref_cache, blocks)[-1:]
    b = new(ids, new_cache, blocks)[-1:]  # paged prefill + slot scatter + device metadata (ours)
    tol = dict(atol=0.06 if dtype == torch.bfloat16 else 0.015, rtol=0.02)
    torch.testing.assert_close(b, a, **tol)
    for pos in range(5, 11):
        token = a.argmax(-1)
        a = ref(token, ref_cache, blocks, pos)
        b = new(token, new_cache, blocks, pos)  # range write + paged decode (ours)
        torch.testing.assert_close(b, a, **tol)
        assert a.argmax() == b.argmax()
    # batched decode: KV append + paged decode for three requests of different lengths
    tables = torch.tensor([[6, 1, 4, 0], [2, 3, -1, -1], [5, 7, -1, -1]], device="cuda")
    for cache, model in ((ref_cache, ref), (new_cache, new)):
        model(torch.tensor([3, 9, 2], device="cuda"), cache, [2, 3], 0)
        model(torch.tensor([4, 4, 1, 2, 2], device="cuda"), cache, [5, 7], 0)
    positions = torch.tensor([11, 3, 5], device="cuda")
    tokens = torch.tensor([7, 8, 9], device="cuda")
    for _ in range(3):
        a = ref.forward_decode_batch(tokens, ref_cache, tables, positions)
        b = new.forward_decode_batch(tokens, new_cache, tables, positions)
        torch.testing.assert_close(b, a, **tol)
        assert torch.equal(a.argmax(-1), b.argmax(-1))
        tokens, positions = a.argmax(-1), positions + 1
    assert _lib.device_status() == 0


def test_reference_decode_graph_bucket_captures_and_replays_installed_ops(cuda_device, reference_engine):
    from mini_engine.engine.cuda_graph import DecodeGraphBucket

    ref, new = _models(reference_engine, torch.float16, seed=11)
    num_blocks, bs = 24, 4
    ref_cache, new_cache = ref.create_cache(num_blocks, bs), new.create_cache(num_blocks, bs)
    gen = torch.Generator(device="cuda").manual_seed(5)
    for cache in (ref_cache, new_cache):  # identical random history in both pools
        cache.key.copy_(torch.randn(cache.key.shape, generator=gen.manual_seed(5), device="cuda").half())
        cache.value.copy_(torch.randn(cache.value.shape, generator=gen.manual_seed(6), device="cuda").half())
    padding = [20, 21, 22, 23]
    bucket = DecodeGraphBucket(new, new_cache, 4, 6, padding_block_ids=padding)
    bucket.capture()
    steps = [([3, 7, 1], [9, 4, 13], [[0, 1, 2], [3, 4], [5, 6, 7, 8]]),
             ([2, 5], [10, 5], [[0, 1, 2], [3, 4]]),
             ([6, 6, 6, 6], [11, 6, 14, 0], [[0, 1, 2], [3, 4], [5, 6, 7, 8], [9]])]
    for tokens, positions, tables in steps:
        logits = bucket.replay_metadata(tokens, positions, tables).clone()
        width = 6
        dense = torch.full((len(tokens), width), -1, dtype=torch.long, device="cuda")
        for row, table in enumerate(tables):
            dense[row, :len(table)] = torch.tensor(table)
        expected = ref.forward_decode_batch(torch.tensor(tokens, device="cuda"), ref_cache, dense,
                                            torch.tensor(positions, device="cuda"))
        torch.testing.assert_close(logits, expected, atol=0.015, rtol=0.02)
        assert torch.equal(logits.argmax(-1), expected.argmax(-1))
    used = sorted({page for _, _, tables in steps for table in tables for page in table})
    for mine, theirs in ((new_cache.key, ref_cache.key), (new_cache.value, ref_cache.value)):
        # layer 0's appended rows come from identical inputs: the KV append must match bit for bit;
        # deeper layers see the attention outputs of the layers before, equal within tolerance
        assert torch.equal(mine[0, used], theirs[0, used])
        torch.testing.assert_close(mine[:, used], theirs[:, used], atol=0.02, rtol=0.02)
    del bucket
    assert _lib.device_status() == 0


def _run_runtime(model, cache, num_blocks, bs, prompts, *, new_tokens, steps):
    from mini_engine.cache import BlockManager
    from mini_engine.engine.request import GenerationRequest
    from mini_engine.engine.runtime import NativeBatchRuntime
    from mini_engine.engine.scheduler import Scheduler

    manager = BlockManager(num_blocks, bs)
    scheduler = Scheduler(manager, max_num_batched_tokens=64)
    runtime = NativeBatchRuntime(model, scheduler, cache, eos_token_ids=[])
    requests = []
    for wave in prompts:
        for name, prompt in wave:
            request = GenerationRequest(name, list(prompt), max_new_tokens=new_tokens)
            scheduler.add_request(request)
            requests.append(request)
        for _ in range(steps):
            runtime.step()
    return {r.request_id: (list(r.output_token_ids), r.prefix_len) for r in requests}


def test_reference_runtime_prefill_prefix_hit_and_decode_on_installed_ops(cuda_device, reference_engine):
    ref, new = _models(reference_engine, torch.float32, seed=21)
    num_blocks, bs = 48, 4
    shared = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 7, 7]  # three complete pages
    prompts = [[("a", shared), ("b", [8, 6, 7, 5, 3, 0, 9])],
               # the second wave hits the pages the first one cached: c and e compute only their
               # suffix chunk over the shared pages, d is an exact hit (cached logits, no prefill)
               [("c", shared + [2, 8]), ("d", list(shared)), ("e", [8, 6, 7, 5, 1])]]
    expected = _run_runtime(ref, ref.create_cache(num_blocks, bs), num_blocks, bs, prompts, new_tokens=4, steps=5)
    actual = _run_runtime(new, new.create_cache(num_blocks, bs), num_blocks, bs, prompts, new_tokens=4, steps=5)
    assert actual == expected
    assert expected["c"][1] == 12 and expected["d"][1] == 12 and expected["e"][1] == 4  # prefix-cache hits
    assert all(len(tokens) == 4 for tokens, _ in expected.values())
    assert _lib.device_status() == 0
