"""Bounded waits give up cleanly: status bit set, kernel ends, nothing left in flight.

``minikv_set_wait_limit`` shortens the limit of the waits in which a producer
waits for its consumers to free a ring slot.  With 100 ns those waits run out
on a large launch (the consumers need microseconds per stage), so the kernel
takes its timeout path: the producer stops issuing and waits for the copies it
already issued, the consumers skip the stages that never arrive, the ticket
protocol of the split-KV merge completes, and the kernel runs to its end.  The
tests check that the status bit is set, that the context stays usable, and that
the next launches with the default limit (and the same workspace, whose ticket
counters must have been left at zero) give the same bits as before.  No wait
here is unbounded and every access stays inside its buffers.
"""

import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.kernels import paged_attention, paged_prefill_attention

pytestmark = pytest.mark.gpu


@pytest.fixture
def short_space_waits(cuda_device):
    assert _lib.device_status() == 0
    yield lambda: _lib.set_wait_limit(100)
    _lib.set_wait_limit(_lib.DEFAULT_WAIT_LIMIT_NS)
    _lib.device_status()  # clear


@pytest.mark.parametrize("dtype,dim", [(torch.float32, 128)])
def test_decode_slot_wait_timeout_sets_status_and_exits_cleanly(short_space_waits, dtype, dim):
    # fp32: the CUDA-core consumers are slower than the copies, so the producer waits for a free
    # slot on every tile and the shortened wait runs out.  (With fp16/bf16 the tensor-core
    # consumers free each slot before the producer has issued the next tile, so those waits
    # never block; the producer and the timeout path are the same code for every dtype.)
    gen = torch.Generator(device="cuda").manual_seed(71)
    batch, context, bs, hq, hkv = 4, 16384, 16, 16, 8
    pages = context // bs
    kc = torch.randn(batch * pages, bs, hkv, dim, device="cuda", generator=gen).to(dtype)
    vc = torch.randn(batch * pages, bs, hkv, dim, device="cuda", generator=gen).to(dtype)
    tables = torch.randperm(batch * pages, device="cuda", generator=gen).view(batch, pages).contiguous()
    lens = torch.full((batch,), context, dtype=torch.int64, device="cuda")
    q = torch.randn(batch, hq, dim, device="cuda", generator=gen).to(dtype)
    good = paged_attention(q, kc, vc, tables, lens, bs, validate=False)
    assert _lib.device_status() == 0
    short_space_waits()
    paged_attention(q, kc, vc, tables, lens, bs, validate=False)
    assert _lib.device_status() & 1, "the shortened slot waits must have run out"
    _lib.set_wait_limit(_lib.DEFAULT_WAIT_LIMIT_NS)
    again = paged_attention(q, kc, vc, tables, lens, bs, validate=False)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(again, good)


def test_prefill_slot_wait_timeout_sets_status_and_exits_cleanly(short_space_waits):
    from myvllm_mini_engine_b200.engine import PrefillBatch

    c = cases.config4()
    bs = c["block_size"]
    batch = PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"], block_size=bs,
                                        num_blocks=c["num_blocks"], device="cuda")
    args = (c["q"].cuda(), c["key_cache"].cuda(), c["value_cache"].cuda(), batch.cu_seqlens_q, batch.query_starts,
            batch.block_tables, batch.context_lens, bs)
    good = paged_prefill_attention(*args, validate=False)
    assert _lib.device_status() == 0
    short_space_waits()
    paged_prefill_attention(*args, validate=False)
    assert _lib.device_status() & 1, "the shortened slot waits must have run out"
    _lib.set_wait_limit(_lib.DEFAULT_WAIT_LIMIT_NS)
    again = paged_prefill_attention(*args, validate=False)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(again, good)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_prefill_wait_timeout_sets_status_and_exits_cleanly(short_space_waits, fmt):
    # The FP8 prefill's producers convert each tile in place before releasing it; with 100 ns their
    # slot waits run out, and the tiles already issued must still land before the CTA exits.
    from myvllm_mini_engine_b200.engine import PrefillBatch
    from myvllm_mini_engine_b200.kernels import paged_prefill_attention_fp8
    from oracle import fp8_kv

    c = cases.config4()
    bs = c["block_size"]
    batch = PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"], block_size=bs,
                                        num_blocks=c["num_blocks"], device="cuda")
    kq = torch.from_numpy(fp8_kv.quantize(c["key_cache"], 0.03, fmt)).cuda()
    vq = torch.from_numpy(fp8_kv.quantize(c["value_cache"], 0.03, fmt)).cuda()
    args = (c["q"].cuda(), kq, vq, batch.cu_seqlens_q, batch.query_starts, batch.block_tables, batch.context_lens,
            bs, 0.03, 0.03)
    good = paged_prefill_attention_fp8(*args, kv_format=fmt, validate=False)
    assert _lib.device_status() == 0
    short_space_waits()
    paged_prefill_attention_fp8(*args, kv_format=fmt, validate=False)
    assert _lib.device_status() & 1, "the shortened waits must have run out"
    _lib.set_wait_limit(_lib.DEFAULT_WAIT_LIMIT_NS)
    again = paged_prefill_attention_fp8(*args, kv_format=fmt, validate=False)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(again, good)
