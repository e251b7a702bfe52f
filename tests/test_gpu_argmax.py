"""Greedy argmax (minikv_argmax_rows) against torch.argmax: the reference's greedy sampler
(mini_engine/sampling.py:14-22) is logits.argmax(dim=-1), so results must be identical,
including ties (lowest index), NaN (counts as the largest) and rows of -inf."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ids(logits):
    from myvllm_mini_engine_b200.engine.qwen3 import greedy_ids

    return greedy_ids(logits)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (5, 1000), (2, 4099), (32, 151936), (256, 151936)])
def test_matches_torch_argmax(cuda_device, dtype, rows, cols):
    gen = torch.Generator(device="cuda").manual_seed(rows * 7919 + cols)
    x = torch.randn(rows, cols, device="cuda", generator=gen).to(dtype)
    assert torch.equal(_ids(x), x.argmax(dim=-1))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ties_nan_and_infinite_rows(cuda_device, dtype):
    cols = 20000
    x = torch.zeros(6, cols, device="cuda", dtype=dtype)
    x[0, [17, 5000, 19999]] = 3.0          # ties: lowest index
    x[1, [9000, 12]] = float("nan")        # NaN counts as the largest: first NaN
    x[1, 3] = 100.0
    x[2].fill_(float("-inf"))              # all -inf: index 0
    x[3, :] = -1.0
    x[3, 15000:] = float("inf")            # +inf ties: first of them
    x[4, 8191] = 1.0                       # on a slice boundary
    x[4, 8192] = 1.0
    x[5, -1] = 1e-3                        # the last column
    assert torch.equal(_ids(x), x.argmax(dim=-1))


def test_strided_rows_and_repeated_calls_in_a_graph(cuda_device):
    base = torch.randn(4, 5003, device="cuda").to(torch.bfloat16)
    x = base[:, :4999]                     # row stride 5003: the scalar path
    want = x.argmax(dim=-1)
    for _ in range(3):                     # the ticket counters are left zero
        assert torch.equal(_ids(x), want)
    y = torch.randn(32, 151936, device="cuda").to(torch.bfloat16)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        _ids(y)  # the stream's workspace exists before capture
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        out = _ids(y)
    for seed in range(3):
        y.copy_(torch.randn(32, 151936, device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed)))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, y.argmax(dim=-1))
