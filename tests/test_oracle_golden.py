"""Pin the CPU oracle to the reference: golden fixtures and literal known answers.

The fixtures under tests/golden were produced by running the reference
engine's own torch paths (make_golden.py); the literal vectors below are the
reference tests' own expectations.  No GPU is needed.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import kv_write, metadata, paged_decode, prefill

GOLDEN = Path(__file__).resolve().parent / "golden"
DECODE = np.load(GOLDEN / "golden_decode.npz")
KV = np.load(GOLDEN / "golden_kv.npz")
PREFILL = np.load(GOLDEN / "golden_prefill.npz")
META = json.loads((GOLDEN / "golden_metadata.json").read_text())
DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def cooked(array, like):
    """Golden raw bits -> tensor of ``like``'s dtype."""
    return torch.from_numpy(np.ascontiguousarray(array)).view(like.dtype).reshape(like.shape)


def decode_args(c):
    return [c[k] for k in ("query", "key_cache", "value_cache", "block_tables", "context_lens")]


@pytest.mark.parametrize("name", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("dim", [16, 32, 80, 128])
def test_decode_oracle_matches_reference_sweep(name, dim):
    c = cases.decode_case(DTYPES[name], head_dim=dim, lengths=(17, 57, 130))
    key = f"sweep_{name}_d{dim}"
    assert cases.sha256_of(decode_args(c)) == str(DECODE[key + "/inputs_sha256"])
    got = paged_decode.paged_attention(*decode_args(c), c["block_size"])
    assert torch.equal(got, cooked(DECODE[key + "/out"], got))


@pytest.mark.parametrize("index,shape", list(enumerate([(4, (1,), 4, 4), (16, (256, 255), 8, 1),
                                                   (32, (257, 1025, 9), 16, 8)])))
def test_decode_oracle_block_and_partition_boundaries(index, shape):
    bs, lengths, heads, kv = shape
    c = cases.decode_case(torch.bfloat16, block_size=bs, lengths=lengths, heads=heads, kv_heads=kv, head_dim=32)
    got = paged_decode.paged_attention(*decode_args(c), bs)
    assert torch.equal(got, cooked(DECODE[f"boundary{index}/out"], got))


@pytest.mark.parametrize("name,build", [("config1", cases.config1), ("config2", cases.config2),
                                        ("config3", cases.config3)])
def test_append_decode_configs_match_reference(name, build):
    c = build()
    inputs = [c[k] for k in ("query", "key_cache", "value_cache", "block_tables", "token_offsets", "key", "value")]
    assert cases.sha256_of(inputs) == str(DECODE[name + "/inputs_sha256"])
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(kc, vc, c["block_tables"], c["token_offsets"], c["key"], c["value"],
                                  c["block_size"])
    assert cases.sha256_of([kc, vc]) == str(DECODE[name + "/caches_sha256"])
    got = paged_decode.paged_attention(c["query"], kc, vc, c["block_tables"], c["context_lens"], c["block_size"])
    assert torch.equal(got, cooked(DECODE[name + "/out"], got))


def test_decode_oracle_matches_reference_make_case_fp32_oracle():
    names = ("query", "key_cache", "value_cache", "block_tables", "context_lens")
    dtypes = (torch.float16, torch.float16, torch.float16, torch.int64, torch.int64)
    tensors = [torch.from_numpy(DECODE["make_case/" + n]).view(t) for n, t in zip(names, dtypes)]
    got = paged_decode.paged_attention_fp32(*tensors, 4)
    torch.testing.assert_close(got, torch.from_numpy(DECODE["make_case/fp32_oracle"]), atol=0, rtol=0)


def test_decode_oracle_rejects_invalid_length_like_fallback():
    c = cases.decode_case(torch.float32, head_dim=16, lengths=(5,))
    c["context_lens"][0] = 0
    with pytest.raises(ValueError, match="invalid context length"):
        paged_decode.paged_attention(*decode_args(c), c["block_size"])


def test_trusted_oracle_masks_invalid_pages_and_lengths():
    c = cases.decode_case(torch.float32, head_dim=16, lengths=(40, 33, 7))
    args = decode_args(c)
    full = paged_decode.paged_attention_fp32(*args, c["block_size"])
    trusted = paged_decode.paged_attention_trusted_fp32(*args, c["block_size"])
    torch.testing.assert_close(trusted, full, atol=1e-6, rtol=1e-6)
    args[3] = args[3].clone()
    args[3].fill_(-1)  # corrupt every page: paged_attention.cu:73-83 -> all-zero rows
    assert not paged_decode.paged_attention_trusted_fp32(*args, c["block_size"]).any()
    args = decode_args(c)
    args[4] = torch.tensor([0, 10_000, 7])  # out-of-range lengths -> zero rows
    out = paged_decode.paged_attention_trusted_fp32(*args, c["block_size"])
    assert not out[:2].any() and out[2].abs().sum() > 0


def test_kv_write_oracles_match_reference():
    c = cases.slots_case()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_slots(kc, vc, c["slot_mapping"], c["key"], c["value"])
    assert torch.equal(kc, cooked(KV["slots/key_cache"], kc)) and torch.equal(vc, cooked(KV["slots/value_cache"], vc))
    c = cases.range_case()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache(kc, vc, c["block_ids"], c["token_offset"], c["key"], c["value"], c["block_size"])
    assert torch.equal(kc, cooked(KV["range/key_cache"], kc)) and torch.equal(vc, cooked(KV["range/value_cache"], vc))
    c = cases.batch_write_case()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    valid = [0, 1, 2]
    kv_write.write_kv_cache_batch(kc, vc, c["block_tables"][valid], c["token_offsets"][valid],
                                  c["key"][valid], c["value"][valid], c["block_size"])
    assert torch.equal(kc, cooked(KV["batch/key_cache"], kc)) and torch.equal(vc, cooked(KV["batch/value_cache"], vc))


def test_batch_write_oracle_skips_invalid_rows():
    c = cases.batch_write_case()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    kv_write.write_kv_cache_batch(kc, vc, c["block_tables"], c["token_offsets"], c["key"], c["value"],
                                  c["block_size"])
    # rows 3 and 4 point at an unallocated page / past the table: identical to valid-only write
    assert torch.equal(kc, cooked(KV["batch/key_cache"], kc)) and torch.equal(vc, cooked(KV["batch/value_cache"], vc))


def test_copy_blocks_oracle_is_page_assignment():
    pool = torch.arange(3 * 6 * 2 * 2 * 4, dtype=torch.float32).view(3, 6, 2, 2, 4)
    vpool = -pool
    expected_k, expected_v = pool.clone(), vpool.clone()
    for src, dst in [(1, 4), (4, 5)]:
        expected_k[:, dst] = expected_k[:, src]
        expected_v[:, dst] = expected_v[:, src]
    kv_write.copy_blocks(pool, vpool, [(1, 4), (4, 5)])
    assert torch.equal(pool, expected_k) and torch.equal(vpool, expected_v)


def test_prefill_oracle_matches_reference():
    c = cases.ragged_small()
    args = [c[k] for k in ("q", "key_cache", "value_cache", "cu_seqlens_q", "query_starts",
                           "block_tables", "context_lens")]
    got = prefill.paged_prefill_attention(*args, c["block_size"])
    assert torch.equal(got, cooked(PREFILL["small/out"], got))
    torch.testing.assert_close(prefill.per_token_fp32(*args, c["block_size"]).to(got.dtype), got,
                               atol=1e-6, rtol=1e-5)  # test_ragged_kernels.py:30-34
    for name in ("fp16", "bf16"):
        c = cases.ragged_prefill_case(DTYPES[name])
        args = [c[k] for k in ("q", "key_cache", "value_cache", "cu_seqlens_q", "query_starts",
                               "block_tables", "context_lens")]
        assert cases.sha256_of(args) == str(PREFILL[f"ragged_{name}/inputs_sha256"])
        got = prefill.paged_prefill_attention(*args, c["block_size"])
        assert torch.equal(got, cooked(PREFILL[f"ragged_{name}/out"], got))


def test_config4_cow_scatter_prefill_oracle_matches_reference():
    c = cases.config4()
    with pytest.raises(ValueError, match="shared by requests"):
        metadata.prefill_metadata(c["tokens"], c["tables"], c["starts"], block_size=c["block_size"],
                                  num_blocks=c["num_blocks"])
    assert str(PREFILL["config4/precow_error"]) == "prefill cannot write a physical page shared by requests"
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    pool_k, pool_v = kc.unsqueeze(0), vc.unsqueeze(0)
    kv_write.copy_blocks(pool_k, pool_v, [c["cow_pair"]])
    meta = metadata.prefill_metadata(c["tokens"], c["cow_tables"], c["starts"], block_size=c["block_size"],
                                     num_blocks=c["num_blocks"])
    t = {k: torch.tensor(v, dtype=torch.int64) for k, v in meta.items()}
    kv_write.write_kv_cache_slots(kc, vc, t["slot_mapping"], c["key"], c["value"])
    assert cases.sha256_of([kc, vc]) == str(PREFILL["config4/caches_sha256"])
    out = prefill.paged_prefill_attention(c["q"], kc, vc, t["cu_seqlens_q"], t["query_starts"],
                                          t["block_tables"], t["context_lens"], c["block_size"])
    rows = torch.from_numpy(PREFILL["config4/rows"])
    assert torch.equal(out[rows], cooked(PREFILL["config4/out_rows"], out[rows]))
    torch.testing.assert_close(out.float().sum(dim=(1, 2)), torch.from_numpy(PREFILL["config4/row_sums"]),
                               atol=0, rtol=0)


def test_metadata_oracle_matches_reference_and_literal_golden():
    g = cases.METADATA_GOLDEN
    got = metadata.prefill_metadata(*g["args"], block_size=g["block_size"], num_blocks=g["num_blocks"])
    for name, values in g["expected"].items():  # test_ragged_model.py:42-53
        assert got[name] == values
    assert got == META["golden"]
    m = cases.metadata_random()
    got = metadata.prefill_metadata(m["tokens"], m["tables"], m["starts"], block_size=m["block_size"],
                                    num_blocks=m["num_blocks"])
    assert got == META["random"]


@pytest.mark.parametrize("index", range(len(cases.METADATA_REJECTIONS)))
def test_metadata_oracle_rejections_match_reference_messages(index):
    tokens, tables, starts, fragment = cases.METADATA_REJECTIONS[index]
    with pytest.raises(ValueError, match=fragment) as error:
        metadata.prefill_metadata(tokens, tables, starts, block_size=4, num_blocks=16)
    assert str(error.value) == META["rejections"][index]


def test_decode_bucket_metadata_padding_rows():
    got = metadata.decode_bucket_metadata([7, 9], [17, 3], [[4, 5], [6]], batch_size=4, max_blocks=3,
                                          padding_pages=[10, 11, 12, 13])
    assert got["input_ids"] == [7, 9, 0, 0] and got["positions"] == [17, 3, 0, 0]
    assert got["block_tables"] == [[4, 5, -1], [6, -1, -1], [12, -1, -1], [13, -1, -1]]


QWEN3 = np.load(GOLDEN / "golden_qwen3.npz")


@pytest.mark.parametrize("name", ["fp32", "bf16"])
def test_decode_step_oracle_matches_reference_model(name):
    """oracle.qwen3.decode_step == NativeQwen3.forward_decode_batch (torch backends, fused projections)."""
    from oracle import qwen3

    dtype = DTYPES[name]
    cfg = cases.qwen3_tiny_config()
    w = cases.qwen3_weights(cfg, dtype, seed=501)
    c = cases.qwen3_decode_case(cfg, dtype, contexts=(5, 11, 2, 16), block_size=4, seed=502)
    key = f"qwen3_{name}"
    inputs = ([c["input_ids"], c["positions"], c["block_tables"], c["key_pool"], c["value_pool"], w.embed]
              + [t for layer in w.layers for t in (layer.qkv, layer.o, layer.gate_up, layer.down)])
    assert cases.sha256_of(inputs) == str(QWEN3[key + "/inputs_sha256"])
    kp, vp = c["key_pool"].clone(), c["value_pool"].clone()
    logits = qwen3.decode_step(cfg, w, c["input_ids"], kp, vp, c["block_tables"], c["positions"])
    assert torch.equal(logits, cooked(QWEN3[key + "/logits"], logits))
    assert torch.equal(kp, cooked(QWEN3[key + "/key_pool"], kp))
    assert torch.equal(vp, cooked(QWEN3[key + "/value_pool"], vp))
    # the step appended exactly one row per request and layer
    changed = (kp != c["key_pool"]).any(dim=-1).any(dim=-1).sum().item()
    assert changed == cfg.num_hidden_layers * len(c["positions"])
