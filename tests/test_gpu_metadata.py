"""Device-side metadata construction: bit-exact against the oracle and the reference's golden values."""

import ctypes
import json
from pathlib import Path

import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.engine import PrefillBatch
from oracle import metadata

pytestmark = pytest.mark.gpu
META = json.loads((Path(__file__).resolve().parent / "golden" / "golden_metadata.json").read_text())
NAMES = ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "query_starts", "context_lens", "block_tables")


def test_prefill_metadata_literal_golden(cuda_device):
    g = cases.METADATA_GOLDEN
    batch = PrefillBatch.from_sequences(*g["args"], block_size=g["block_size"], num_blocks=g["num_blocks"],
                                        device="cuda")
    for name, values in g["expected"].items():  # tests/test_ragged_model.py:42-53
        assert getattr(batch, name).tolist() == values
    assert {n: getattr(batch, n).tolist() for n in NAMES} == META["golden"]
    assert batch.query_lengths == (3, 2) and batch.query_offsets == (0, 3, 5) and batch.starts == (4, 4)
    assert batch.block_ids == ((3, 1), (3, 2)) and batch.num_tokens == 5 and batch.batch_size == 2


def test_prefill_metadata_random_batch_matches_reference(cuda_device):
    m = cases.metadata_random()
    batch = PrefillBatch.from_sequences(m["tokens"], m["tables"], m["starts"], block_size=m["block_size"],
                                        num_blocks=m["num_blocks"], device="cuda")
    assert {n: getattr(batch, n).tolist() for n in NAMES} == META["random"]
    expected = metadata.prefill_metadata(m["tokens"], m["tables"], m["starts"], block_size=m["block_size"],
                                         num_blocks=m["num_blocks"])
    assert {n: getattr(batch, n).tolist() for n in NAMES} == expected
    batch.validate(block_size=m["block_size"], num_blocks=m["num_blocks"], device=cuda_device,
                   max_position_embeddings=4096, vocab_size=151936)
    with pytest.raises(ValueError, match="vocabulary"):
        batch.validate(block_size=m["block_size"], num_blocks=m["num_blocks"], device=cuda_device,
                       max_position_embeddings=4096, vocab_size=10)


def test_decode_bucket_tables_match_oracle_and_work_inside_a_graph(cuda_device):
    lib = _lib.load()
    batch_size, max_blocks = 6, 5
    padding = torch.tensor([40, 41, 42, 43, 44, 45], device="cuda")
    cap = batch_size * max_blocks
    staged = torch.zeros(1 + 3 * batch_size + 1 + cap, dtype=torch.int64, device="cuda")
    ids = torch.empty(batch_size, dtype=torch.int64, device="cuda")
    pos = torch.empty_like(ids)
    tables = torch.empty(batch_size, max_blocks, dtype=torch.int64, device="cuda")
    view = lambda a, n: staged.narrow(0, a, n)  # noqa: E731
    active, tokens, positions = view(0, 1), view(1, batch_size), view(1 + batch_size, batch_size)
    cu, blocks = view(1 + 2 * batch_size, batch_size + 1), view(2 + 3 * batch_size, cap)

    def stage(tok, posn, rows):
        flat = [p for row in rows for p in row]
        cu_host = [0]
        for row in rows:
            cu_host.append(cu_host[-1] + len(row))
        active.fill_(len(tok))
        tokens[:len(tok)].copy_(torch.tensor(tok))
        positions[:len(tok)].copy_(torch.tensor(posn))
        cu[:len(cu_host)].copy_(torch.tensor(cu_host))
        blocks[:len(flat)].copy_(torch.tensor(flat))

    def launch():
        rc = lib.minikv_build_decode_tables(active.data_ptr(), tokens.data_ptr(), positions.data_ptr(),
                                            cu.data_ptr(), blocks.data_ptr(), padding.data_ptr(), batch_size,
                                            max_blocks, ids.data_ptr(), pos.data_ptr(), tables.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "build_decode_tables")

    stage([7, 9], [17, 3], [[4, 5], [6]])
    launch()
    graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        launch()
    for tok, posn, rows in (([7, 9], [17, 3], [[4, 5], [6]]), ([1, 2, 3], [0, 80, 9], [[1], [2, 3, 4, 5, 8], [9]])):
        stage(tok, posn, rows)
        graph.replay()
        expected = metadata.decode_bucket_metadata(tok, posn, rows, batch_size=batch_size, max_blocks=max_blocks,
                                                   padding_pages=padding.tolist())
        assert ids.tolist() == expected["input_ids"] and pos.tolist() == expected["positions"]
        assert tables.tolist() == expected["block_tables"]
