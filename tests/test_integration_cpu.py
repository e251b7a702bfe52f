"""The drop-in installer, checked on the host against the reference engine package.

Needs the copy of the reference engine under baseline/_ref (skipped without
it).  No kernel runs here: name binding, backend routing (a CUDA backend
reaches this package, the reference's "torch" backend still runs the
reference's own function) and the copy-on-write methods added to the
reference allocator.  The GPU half is tests/test_gpu_integration.py.
"""

import torch

from myvllm_mini_engine_b200 import integration, kernels
from myvllm_mini_engine_b200.engine import PrefillBatch


def test_install_routes_cuda_backends_of_every_reference_entry_point(reference_engine):
    import mini_engine.engine.batch as batch
    import mini_engine.engine.runtime as runtime
    import mini_engine.kernels.data as data
    import mini_engine.kernels.paged as paged
    import mini_engine.kernels.prefill as prefill
    import mini_engine.model.native_qwen3 as nq

    original = data.write_kv_cache_batch
    patched = integration.install(reference_engine)
    assert integration.install(reference_engine) == patched  # idempotent: no wrapper around a wrapper
    for module, name, ours in ((paged, "paged_attention", kernels.paged_attention),
                               (data, "write_kv_cache", kernels.write_kv_cache),
                               (data, "write_kv_cache_batch", kernels.write_kv_cache_batch),
                               (data, "write_kv_cache_slots", kernels.write_kv_cache_slots),
                               (prefill, "paged_prefill_attention", kernels.paged_prefill_attention)):
        assert getattr(module, name).__minikv_ours__ is ours
    assert nq.paged_attention is paged.paged_attention and nq.write_kv_cache_batch is data.write_kv_cache_batch
    assert nq.write_kv_cache_slots is data.write_kv_cache_slots
    assert nq.paged_prefill_attention is prefill.paged_prefill_attention
    assert batch.PrefillBatch is PrefillBatch and runtime.PrefillBatch is PrefillBatch
    assert data.write_kv_cache_batch.__minikv_reference__ is original
    assert data.write_kv_cache_batch.__kwdefaults__["backend"] == "torch"  # the reference default is kept
    assert nq.Attention.forward_decode_batch.__minikv_reference__ is not None  # append + decode fused
    assert len(patched) >= 15


def test_installed_ops_keep_the_reference_torch_path(reference_engine):
    import mini_engine.kernels.data as data
    import mini_engine.kernels.paged as paged

    integration.install(reference_engine)
    gen = torch.Generator().manual_seed(3)
    kc = torch.zeros(4, 4, 2, 16)
    vc = torch.zeros_like(kc)
    key, value = torch.randn(2, 2, 16, generator=gen), torch.randn(2, 2, 16, generator=gen)
    tables = torch.tensor([[2, 0], [1, 3]])
    offsets = torch.tensor([5, 0])
    data.write_kv_cache_batch(kc, vc, tables, offsets, key, value, 4)  # default backend: the reference's torch
    assert torch.equal(kc[0, 1], key[0]) and torch.equal(vc[1, 0], value[1])
    query = torch.randn(2, 4, 16, generator=gen)
    out = paged.paged_attention(query, kc, vc, tables, offsets + 1, 4, backend="torch")
    assert out.shape == query.shape and torch.isfinite(out).all()
    try:  # a CUDA backend reaches this package, which has no CPU path
        paged.paged_attention(query, kc, vc, tables, offsets + 1, 4, backend="cuda")
    except RuntimeError as error:
        assert "query must be CUDA" in str(error)
    else:
        raise AssertionError("the cuda backend must run this package's kernels")


def test_install_adds_copy_on_write_to_the_reference_allocator(reference_engine):
    from mini_engine.cache.block_manager import BlockManager
    from mini_engine.cache.kv_cache import KVCachePool

    integration.install(reference_engine)
    manager = BlockManager(8, 4)
    shared = manager.allocate("a", 8)
    manager.attach("b", shared)
    (src, dst), = manager.prepare_write("b", 6, 8)
    assert src == shared[1] and manager.table("b").block_ids == (shared[0], dst)
    assert manager.copy_on_write("b", 1) is None
    assert hasattr(KVCachePool, "copy_blocks")
