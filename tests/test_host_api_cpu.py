"""Host-side contract of the drop-in API, checked without a GPU.

Mirrors the reference's CPU-runnable tests for the same entry points
(tests/test_ragged_kernels.py:48-99, tests/test_ragged_model.py:56-73,
tests/test_cuda_paged_attention.py:58-70): argument and metadata errors are
raised on the host before any device work.
"""

import pytest
import torch

import cases
from myvllm_mini_engine_b200.cache import copy_on_write, prepare_write
from myvllm_mini_engine_b200.engine import PrefillBatch
from myvllm_mini_engine_b200.kernels import (copy_blocks, paged_attention, paged_prefill_attention,
                                             write_kv_cache, write_kv_cache_batch, write_kv_cache_slots)


def test_decode_requires_cuda_backend_and_cuda_tensors():
    c = cases.decode_case(torch.float16, head_dim=16, lengths=(5,))
    args = [c[k] for k in ("query", "key_cache", "value_cache", "block_tables", "context_lens")]
    with pytest.raises(ValueError, match="no torch/CPU path"):
        paged_attention(*args, c["block_size"], backend="torch")
    with pytest.raises(RuntimeError, match="query must be CUDA"):
        paged_attention(*args, c["block_size"])


def test_slot_scatter_rejects_races_overlap_and_capacity_before_dispatch():
    c = cases.slots_case()
    key, value, slots = c["key_cache"], c["value_cache"], c["slot_mapping"]
    with pytest.raises(ValueError, match="duplicate"):
        write_kv_cache_slots(key, value, torch.zeros(8, dtype=torch.int64), c["key"], c["value"])
    with pytest.raises(ValueError, match="overlap"):
        write_kv_cache_slots(key, value, slots, key.view(-1, 2, 16)[:8], c["value"])
    with pytest.raises(ValueError, match="overlap"):
        write_kv_cache_slots(key, key, slots, c["key"], c["value"])
    before = key.clone()
    for slot in (-1, 32):
        with pytest.raises(ValueError, match="capacity"):
            write_kv_cache_slots(key, value, torch.tensor([slot]), torch.ones(1, 2, 16), torch.ones(1, 2, 16))
    assert torch.equal(key, before)
    with pytest.raises(ValueError, match="int64"):
        write_kv_cache_slots(key, value, slots.int(), c["key"], c["value"])
    with pytest.raises(ValueError, match="data backend"):
        write_kv_cache_slots(key, value, slots, c["key"], c["value"], backend="torch")


def test_kv_write_shape_errors():
    c = cases.range_case()
    with pytest.raises(ValueError, match="capacity"):
        write_kv_cache(c["key_cache"], c["value_cache"], c["block_ids"], 6, c["key"], c["value"], 4)
    with pytest.raises(ValueError, match="kv_heads, head_dim"):
        write_kv_cache(c["key_cache"], c["value_cache"], c["block_ids"], 0, c["key"][0], c["value"][0], 4)
    c = cases.batch_write_case()
    with pytest.raises(ValueError, match="offset shape"):
        write_kv_cache_batch(c["key_cache"], c["value_cache"], c["block_tables"][:2], c["token_offsets"],
                             c["key"], c["value"], c["block_size"])
    pool = torch.zeros(2, 4, 4, 2, 8)
    with pytest.raises(ValueError, match="CUDA"):
        copy_blocks(pool, pool.clone(), [(0, 1)])


@pytest.mark.parametrize("change,message", [
    (lambda a: a[3].fill_(0), "offset"),
    (lambda a: a[4].fill_(-1), "context"),
    (lambda a: a[6].fill_(99), "capacity"),
    (lambda a: a[5].fill_(-1), "physical"),
    (lambda a: a[5].fill_(8), "physical"),
    (lambda a: a.__setitem__(3, a[3].to(torch.int32)), "int64"),
])
def test_invalid_paged_prefill_metadata_rejected_before_dispatch(change, message):
    c = cases.ragged_small()
    args = [c[k] for k in ("q", "key_cache", "value_cache", "cu_seqlens_q", "query_starts",
                           "block_tables", "context_lens")]
    change(args)
    with pytest.raises(ValueError, match=message):
        paged_prefill_attention(*args, 4)


@pytest.mark.parametrize("index", range(len(cases.METADATA_REJECTIONS)))
def test_prefill_batch_rejections_match_reference(index):
    tokens, tables, starts, fragment = cases.METADATA_REJECTIONS[index]
    with pytest.raises(ValueError, match=fragment):
        PrefillBatch.from_sequences(tokens, tables, starts, block_size=4, num_blocks=16, device="cpu")


def test_prefill_batch_rejects_write_into_shared_page_until_copy_on_write():
    c = cases.config4()
    with pytest.raises(ValueError, match="shared by requests"):
        PrefillBatch.from_sequences(c["tokens"], c["tables"], c["starts"], block_size=c["block_size"],
                                    num_blocks=c["num_blocks"], device="cpu")
    with pytest.raises(ValueError, match="CUDA device"):  # valid after CoW; only the device is missing
        PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"], block_size=c["block_size"],
                                    num_blocks=c["num_blocks"], device="cpu")


# ------------------------------------------- copy-on-write on the reference allocator
def test_copy_on_write_forks_only_shared_pages_of_the_reference_allocator(reference_engine):
    from mini_engine.cache.block_manager import BlockManager

    manager = BlockManager(128, 16)
    shared = manager.allocate("prefix-owner", 512)
    manager.pin(shared)                                   # prefix-cache pin
    for r in range(8):
        manager.attach(f"r{r}", shared)
        manager.grow(f"r{r}", 512 + 128)
    assert manager.refcount(shared[31]) == 10
    free_before = manager.free_blocks
    pairs = prepare_write(manager, "r3", 496, 624)        # chunk starts inside shared page 31
    assert len(pairs) == 1 and pairs[0][0] == shared[31]
    dst = pairs[0][1]
    assert manager.table("r3").block_ids[31] == dst and manager.refcount(dst) == 1
    assert manager.free_blocks == free_before - 1
    assert manager.refcount(shared[31]) == 9 and manager.table("r2").block_ids[31] == shared[31]
    assert prepare_write(manager, "r3", 496, 624) == []  # already private
    assert prepare_write(manager, "r4", 512, 640) == []  # writes only private pages
    assert prepare_write(manager, "r4", 0, 0) == []
    manager.release("r3")                                 # the reference's own release sees the fork
    assert manager.refcount(dst) == 0 and manager.refcount(shared[31]) == 9
    manager.release("prefix-owner")
    manager.unpin(shared)
    for r in (0, 1, 2, 4, 5, 6, 7):
        manager.release(f"r{r}")
    assert manager.free_blocks == 128                     # every page, forked or not, back on the free list


def test_copy_on_write_errors_leave_the_reference_allocator_unchanged(reference_engine):
    from mini_engine.cache.block_manager import BlockManager

    manager = BlockManager(3, 4)
    shared = manager.allocate("a", 8)
    manager.attach("b", shared)
    manager.allocate("c", 4)                              # the last free page
    with pytest.raises(KeyError):
        copy_on_write(manager, "missing", 0)
    with pytest.raises(IndexError):
        copy_on_write(manager, "b", 2)
    with pytest.raises(ValueError):
        prepare_write(manager, "b", 5, 4)
    with pytest.raises(MemoryError):
        copy_on_write(manager, "b", 0)
    assert manager.table("b").block_ids == tuple(shared) and manager.refcount(shared[0]) == 2
    assert copy_on_write(manager, "c", 0) is None         # private page: nothing to fork
