"""The no-allocation decode entry point agrees with the regular one.

minikv_paged_decode_noalloc serves callers that cannot allocate device memory
at call time (a graph capture under a framework that owns all allocations, a
serving loop that bans cudaMalloc after start-up, a cgo/JNI host without a
device allocator).  Its scratch is a built-in device array shared by every
call, which keeps the previous call's contents, so this test calls it twice in
a row -- with a different batch the second time -- and compares each result
with minikv_paged_decode's (caller workspace) within the bf16 tolerance used by
the other decode tests.  The file is named to be collected last; it also runs
on its own in a fresh process.
"""

import ctypes

import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.kernels import paged_attention

pytestmark = pytest.mark.gpu
TOL = 1e-2  # bf16 tolerance of the decode parity tests


def call_noalloc(lib, c, out):
    q, kc = c["query"], c["key_cache"]
    batch, heads, dim = q.shape
    num_blocks, block_size, kv_heads, _ = kc.shape
    return lib.minikv_paged_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), c["value_cache"].data_ptr(), c["block_tables"].data_ptr(),
        c["context_lens"].data_ptr(), out.data_ptr(), batch, heads, kv_heads, dim, num_blocks, block_size,
        c["block_tables"].shape[1], _lib.BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_decode_matches_workspace_decode_on_two_calls_in_a_row(cuda_device):
    lib = _lib.load()
    first = cases.decode_case(torch.bfloat16, lengths=(17, 257, 521, 1030), seed=5)
    second = cases.decode_case(torch.bfloat16, lengths=(300, 9), seed=6)
    for c in (first, second):
        g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
        out = torch.empty_like(g["query"])
        rc = call_noalloc(lib, g, out)
        assert rc == _lib.OK, lib.minikv_last_error().decode()
        expected = paged_attention(g["query"], g["key_cache"], g["value_cache"], g["block_tables"],
                                   g["context_lens"], g["block_size"], validate=False)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), expected.float(), atol=TOL, rtol=TOL)
    assert _lib.device_status() == 0


def test_noalloc_decode_rejects_shapes_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    # 4096 requests x 2 partial records of 16 heads x 256 dims in fp32 exceed the 16 MiB buffer
    q = torch.zeros(4096, 16, 256, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(8, 16, 8, 256, dtype=torch.bfloat16, device="cuda")
    tables = torch.zeros(4096, 1, dtype=torch.int64, device="cuda")
    lens = torch.ones(4096, dtype=torch.int64, device="cuda")
    out = torch.empty_like(q)
    rc = lib.minikv_paged_decode_noalloc(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), tables.data_ptr(),
                                         lens.data_ptr(), out.data_ptr(), 4096, 16, 8, 256, 8, 16, 1,
                                         _lib.BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.EINVAL
    assert "built-in buffer" in lib.minikv_last_error().decode()
