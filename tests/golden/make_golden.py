"""Generate golden fixtures by running the REFERENCE implementation's torch paths.

Usage (build container only; the reference is not available on the GPU box):

    python tests/golden/make_golden.py --reference /path/to/mini-engine-checkout

The reference package writes ``build/`` and ``.cache/`` next to itself when
imported (``mini_engine/runtime.py:8-29``), so it is imported from a private
copy under ``baseline/_ref`` (git-ignored), never from a read-only checkout.

Fixtures written next to this file:
  * ``golden_decode.npz``   -- ``kernels/paged.py`` (backend="torch") and
    ``kernels/data.py::write_kv_cache_batch`` on the cases of ``cases.py``,
    plus ``benchmarks/compare_paged_backends.py::make_case``/``fp32_oracle``;
  * ``golden_kv.npz``       -- ``write_kv_cache``, ``write_kv_cache_batch`` and
    ``write_kv_cache_slots`` (torch paths);
  * ``golden_prefill.npz``  -- ``kernels/prefill.py::paged_prefill_attention``
    (backend="torch"), including BASELINE config 4 (subsampled rows);
  * ``golden_metadata.json`` -- ``engine/batch.py::PrefillBatch.from_sequences``;
  * ``golden_qwen3.npz``    -- ``model/native_qwen3.py::NativeQwen3.forward_decode_batch``
    (all backends torch, projections fused) on a small Qwen3-family model.
Raw bit patterns are stored for fp16/bf16 tensors (as int16).
"""

from __future__ import annotations

import argparse
import json
import shutil
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

_RAW = {torch.float32: torch.int32, torch.float16: torch.int16, torch.bfloat16: torch.int16,
        torch.int64: torch.int64}
DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def raw(t):
    return t.contiguous().view(_RAW[t.dtype]).numpy().copy()


def load_reference(reference: Path):
    """Import the reference engine from ``baseline/_ref`` and its benchmarks from ``reference``.

    ``baseline/_ref`` is the pip install of the reference
    (``python -m pip install --no-index --no-build-isolation --no-deps --target
    baseline/_ref <copy of the reference>``); when it is missing, the reference
    tree is copied there instead.  The ``benchmarks`` package is not part of the
    install and is imported read-only from ``reference`` (no bytecode written).
    """
    copy = REPO / "baseline" / "_ref"
    if not (copy / "mini_engine").is_dir():
        shutil.copytree(reference, copy, ignore=shutil.ignore_patterns(".git"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(copy))
    sys.path.append(str(reference))
    import mini_engine  # noqa: F401  (runs configure_local_cache inside the copy)
    from mini_engine.kernels import data, paged, prefill
    from mini_engine.engine.batch import PrefillBatch
    from benchmarks import compare_paged_backends
    return paged, data, prefill, PrefillBatch, compare_paged_backends


def decode_fixtures(paged, data, compare):
    out = {}
    sweep = [(name, dim) for name in ("fp32", "fp16", "bf16") for dim in (16, 32, 80, 128)]
    for name, dim in sweep:
        c = cases.decode_case(DTYPES[name], head_dim=dim, lengths=(17, 57, 130))
        args = [c[k] for k in ("query", "key_cache", "value_cache", "block_tables", "context_lens")]
        key = f"sweep_{name}_d{dim}"
        out[key + "/inputs_sha256"] = np.array(cases.sha256_of(args))
        out[key + "/out"] = raw(paged.paged_attention(*args, c["block_size"], backend="torch"))
    boundary = [(4, (1,), 4, 4), (16, (256, 255), 8, 1), (32, (257, 1025, 9), 16, 8)]
    for i, (bs, lengths, heads, kv) in enumerate(boundary):  # test_cuda_paged_attention.py:47-55
        c = cases.decode_case(torch.bfloat16, block_size=bs, lengths=lengths, heads=heads,
                              kv_heads=kv, head_dim=32)
        args = [c[k] for k in ("query", "key_cache", "value_cache", "block_tables", "context_lens")]
        out[f"boundary{i}/inputs_sha256"] = np.array(cases.sha256_of(args))
        out[f"boundary{i}/out"] = raw(paged.paged_attention(*args, bs, backend="torch"))
    for name, build in (("config1", cases.config1), ("config2", cases.config2), ("config3", cases.config3)):
        c = build()
        inputs = [c[k] for k in ("query", "key_cache", "value_cache", "block_tables",
                                 "token_offsets", "key", "value")]
        out[name + "/inputs_sha256"] = np.array(cases.sha256_of(inputs))
        kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
        data.write_kv_cache_batch(kc, vc, c["block_tables"], c["token_offsets"], c["key"], c["value"],
                                  c["block_size"], backend="torch")
        out[name + "/caches_sha256"] = np.array(cases.sha256_of([kc, vc]))
        result = paged.paged_attention(c["query"], kc, vc, c["block_tables"], c["context_lens"],
                                       c["block_size"], backend="torch")
        out[name + "/out"] = raw(result)
    # benchmarks/compare_paged_backends.py:32-72 -- the reference's own case + fp32 oracle
    tensors, manifest = compare.make_case(3, 11, heads=4, kv_heads=2, head_dim=16, block_size=4)
    for name in compare.TENSOR_NAMES:
        out["make_case/" + name] = raw(tensors[name])
    out["make_case/fp32_oracle"] = compare.fp32_oracle(tensors, 4).numpy()
    out["make_case/case_sha256"] = np.array(manifest["case_sha256"])
    return out


def kv_fixtures(data):
    out = {}
    c = cases.slots_case()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    data.write_kv_cache_slots(kc, vc, c["slot_mapping"], c["key"], c["value"])
    out["slots/key_cache"], out["slots/value_cache"] = raw(kc), raw(vc)
    c = cases.range_case()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    data.write_kv_cache(kc, vc, c["block_ids"], c["token_offset"], c["key"], c["value"],
                        c["block_size"], backend="torch")
    out["range/key_cache"], out["range/value_cache"] = raw(kc), raw(vc)
    c = cases.batch_write_case()
    valid = [0, 1, 2]  # the torch path has no trusted-mode guards; feed it valid rows only
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    data.write_kv_cache_batch(kc, vc, c["block_tables"][valid], c["token_offsets"][valid],
                              c["key"][valid], c["value"][valid], c["block_size"], backend="torch")
    out["batch/key_cache"], out["batch/value_cache"] = raw(kc), raw(vc)
    return out


def prefill_fixtures(prefill, data, PrefillBatch):
    out = {}
    c = cases.ragged_small()
    args = [c[k] for k in ("q", "key_cache", "value_cache", "cu_seqlens_q", "query_starts",
                           "block_tables", "context_lens")]
    out["small/out"] = raw(prefill.paged_prefill_attention(*args, c["block_size"], backend="torch"))
    for name in ("fp16", "bf16"):
        c = cases.ragged_prefill_case(DTYPES[name])
        args = [c[k] for k in ("q", "key_cache", "value_cache", "cu_seqlens_q", "query_starts",
                               "block_tables", "context_lens")]
        out[f"ragged_{name}/inputs_sha256"] = np.array(cases.sha256_of(args))
        out[f"ragged_{name}/out"] = raw(prefill.paged_prefill_attention(*args, c["block_size"], backend="torch"))
    # CoW of the shared page, scatter of the chunk K/V, paged prefill.
    c = cases.config4()
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    src, dst = c["cow_pair"]
    kc[dst], vc[dst] = kc[src], vc[src]
    batch = PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"],
                                        block_size=c["block_size"], num_blocks=c["num_blocks"], device="cpu")
    data.write_kv_cache_slots(kc, vc, batch.slot_mapping, c["key"], c["value"], backend="torch")
    out["config4/caches_sha256"] = np.array(cases.sha256_of([kc, vc]))
    result = prefill.paged_prefill_attention(c["q"], kc, vc, batch.cu_seqlens_q, batch.query_starts,
                                             batch.block_tables, batch.context_lens, c["block_size"],
                                             backend="torch")
    out["config4/rows"] = np.arange(0, result.shape[0], 16)
    out["config4/out_rows"] = raw(result[::16])
    out["config4/row_sums"] = result.float().sum(dim=(1, 2)).numpy()
    try:
        PrefillBatch.from_sequences(c["tokens"], c["tables"], c["starts"], block_size=c["block_size"],
                                    num_blocks=c["num_blocks"], device="cpu")
        out["config4/precow_error"] = np.array("")
    except ValueError as error:
        out["config4/precow_error"] = np.array(str(error))
    return out


def qwen3_fixtures():
    """NativeQwen3.forward_decode_batch (native_qwen3.py:423-456), all backends torch, projections fused."""
    from mini_engine.model.native_qwen3 import NativeQwen3, Qwen3Config

    out = {}
    cfg = cases.qwen3_tiny_config()
    ref_cfg = Qwen3Config(**{k: getattr(cfg, k) for k in Qwen3Config.__dataclass_fields__ if hasattr(cfg, k)})
    for name in ("fp32", "bf16"):
        dtype = DTYPES[name]
        w = cases.qwen3_weights(cfg, dtype, seed=501)
        model = NativeQwen3(ref_cfg, prefill_backend="math", decode_backend="torch", elementwise_backend="torch",
                            data_backend="torch", linear_backend="torch")
        q_rows, kv_rows = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
        state = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.norm, "lm_head.weight": w.embed}
        for i, layer in enumerate(w.layers):
            p = f"model.layers.{i}."
            state[p + "self_attn.q_proj.weight"] = layer.qkv[:q_rows]
            state[p + "self_attn.k_proj.weight"] = layer.qkv[q_rows:q_rows + kv_rows]
            state[p + "self_attn.v_proj.weight"] = layer.qkv[q_rows + kv_rows:]
            state[p + "self_attn.o_proj.weight"] = layer.o
            state[p + "self_attn.q_norm.weight"] = layer.q_norm
            state[p + "self_attn.k_norm.weight"] = layer.k_norm
            state[p + "mlp.gate_proj.weight"] = layer.gate_up[:cfg.intermediate_size]
            state[p + "mlp.up_proj.weight"] = layer.gate_up[cfg.intermediate_size:]
            state[p + "mlp.down_proj.weight"] = layer.down
            state[p + "input_layernorm.weight"] = layer.input_norm
            state[p + "post_attention_layernorm.weight"] = layer.post_norm
        model = model.to(dtype)
        model.load_state_dict({k: v.clone() for k, v in state.items()}, strict=True)
        model.enable_projection_fusion()
        c = cases.qwen3_decode_case(cfg, dtype, contexts=(5, 11, 2, 16), block_size=4, seed=502)
        cache = model.create_cache(c["key_pool"].shape[1], c["block_size"])
        cache.key.copy_(c["key_pool"])
        cache.value.copy_(c["value_pool"])
        logits = model.forward_decode_batch(c["input_ids"], cache, c["block_tables"], c["positions"])
        key = f"qwen3_{name}"
        out[key + "/inputs_sha256"] = np.array(cases.sha256_of(
            [c["input_ids"], c["positions"], c["block_tables"], c["key_pool"], c["value_pool"], w.embed]
            + [t for layer in w.layers for t in (layer.qkv, layer.o, layer.gate_up, layer.down)]))
        out[key + "/logits"] = raw(logits)
        out[key + "/key_pool"] = raw(cache.key)
        out[key + "/value_pool"] = raw(cache.value)
    return out


def metadata_fixtures(PrefillBatch):
    names = ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "query_starts",
             "context_lens", "block_tables")

    def run(tokens, tables, starts, block_size, num_blocks):
        batch = PrefillBatch.from_sequences(tokens, tables, starts, block_size=block_size,
                                            num_blocks=num_blocks, device="cpu")
        return {name: getattr(batch, name).tolist() for name in names}

    result = {}
    g = cases.METADATA_GOLDEN
    result["golden"] = run(*g["args"], g["block_size"], g["num_blocks"])
    m = cases.metadata_random()
    result["random"] = run(m["tokens"], m["tables"], m["starts"], m["block_size"], m["num_blocks"])
    errors = []
    for tokens, tables, starts, _ in cases.METADATA_REJECTIONS:
        try:
            PrefillBatch.from_sequences(tokens, tables, starts, block_size=4, num_blocks=16, device="cpu")
            errors.append("")
        except ValueError as error:
            errors.append(str(error))
    result["rejections"] = errors
    return result


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, required=True,
                        help="a checkout of the reference engine (copied to baseline/_ref)")
    args = parser.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    paged, data, prefill, PrefillBatch, compare = load_reference(args.reference)
    np.savez_compressed(HERE / "golden_decode.npz", **decode_fixtures(paged, data, compare))
    np.savez_compressed(HERE / "golden_kv.npz", **kv_fixtures(data))
    np.savez_compressed(HERE / "golden_prefill.npz", **prefill_fixtures(prefill, data, PrefillBatch))
    np.savez_compressed(HERE / "golden_qwen3.npz", **qwen3_fixtures())
    (HERE / "golden_metadata.json").write_text(json.dumps(metadata_fixtures(PrefillBatch)))
    for path in sorted(HERE.glob("golden_*")):
        print(f"{path.name}: {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
