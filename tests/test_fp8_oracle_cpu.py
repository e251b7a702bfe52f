"""FP8 KV pool: the oracle pinned against torch's float8_e4m3fn, and the C-ABI argument checks (no GPU)."""

import numpy as np
import pytest
import torch

from myvllm_mini_engine_b200 import _lib
from oracle import fp8_kv


TORCH_DTYPES = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2}


def torch_fp8(values, fmt="e4m3"):
    vmax = fp8_kv.FORMATS[fmt][3]
    clipped = np.clip(values, -vmax, vmax)
    return torch.from_numpy(clipped).to(TORCH_DTYPES[fmt]).view(torch.uint8).numpy()


def torch_e4m3(values):
    return torch_fp8(values, "e4m3")


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_encoder_matches_torch_on_every_bf16_value(fmt):
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    finite = np.isfinite(x)
    assert np.array_equal(fp8_kv.encode_fp8(x, fmt)[finite], torch_fp8(x[finite], fmt))


def test_e5m2_encoder_on_random_fp32_and_edges():
    gen = np.random.default_rng(12)
    x = (gen.standard_normal(500_000) * gen.choice([1e-6, 0.01, 1.0, 500.0, 3e4], 500_000)).astype(np.float32)
    assert np.array_equal(fp8_kv.encode_fp8(x, "e5m2"), torch_fp8(x, "e5m2"))
    edges = np.array([np.inf, -np.inf, -0.0, 2 ** -17, 3 * 2 ** -17, 61440.0], dtype=np.float32)
    assert fp8_kv.encode_fp8(edges, "e5m2").tolist() == [0x7B, 0xFB, 0x80, 0x00, 0x02, 0x7B]


def test_encoder_matches_torch_on_random_fp32_and_edges():
    gen = np.random.default_rng(11)
    x = (gen.standard_normal(500_000) * gen.choice([1e-4, 0.01, 1.0, 50.0, 400.0], 500_000)).astype(np.float32)
    assert np.array_equal(fp8_kv.encode_e4m3(x), torch_e4m3(x))
    edges = np.array([np.inf, -np.inf, np.nan, -0.0, 2 ** -10, 3 * 2 ** -10, 464.0, 1e30], dtype=np.float32)
    assert fp8_kv.encode_e4m3(edges).tolist() == [0x7E, 0xFE, 0x7F, 0x80, 0x00, 0x02, 0x7E, 0x7E]


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_decode_table_matches_torch(fmt):
    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes).view(TORCH_DTYPES[fmt]).float().numpy()
    got = fp8_kv.decode_fp8(codes, fmt)
    nan = np.isnan(want)
    assert np.array_equal(nan, np.isnan(got)) and np.array_equal(got[~nan], want[~nan])
    # every finite code survives encode(decode(code)) unchanged
    finite = np.isfinite(want)
    assert np.array_equal(fp8_kv.encode_fp8(got[finite], fmt), codes[finite])


def test_scatter_oracle_skips_slots_outside_the_capacity():
    kc = torch.zeros(2, 4, 1, 16, dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    key = torch.ones(3, 1, 16)
    slots = torch.tensor([1, -1, 8])
    fp8_kv.scatter_slots_fp8(kc, vc, slots, key, -key, 0.5, 0.25)
    assert kc.view(-1, 16)[1].tolist() == [fp8_kv.encode_e4m3(np.float32(2.0)).item()] * 16
    assert vc.view(-1, 16)[1].tolist() == [fp8_kv.encode_e4m3(np.float32(-4.0)).item()] * 16
    assert int(kc.sum()) == 16 * int(kc.view(-1, 16)[1, 0])


def test_abi_rejects_bad_fp8_arguments_without_a_gpu():
    lib = _lib.load()
    p = 16  # never dereferenced: every call below fails its checks first
    rc = lib.minikv_paged_decode_fp8(p, p, p, p, p, p, p, 1 << 20, 2, 8, 4, 80, 10, 16, 4, 0.1, 0.1, 0, _lib.BF16, None)
    assert rc == _lib.EINVAL and "head_dim" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode_fp8(p, p, p, p, p, p, p, 1 << 20, 2, 8, 4, 128, 10, 16, 4, 0.1, 0.1, 0, _lib.F32, None)
    assert rc == _lib.EINVAL and "FP16/BF16" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode_fp8(p, p, p, p, p, p, p, 1 << 20, 2, 8, 4, 128, 10, 16, 4, 0.0, 0.1, 0, _lib.BF16, None)
    assert rc == _lib.EINVAL and "scales" in lib.minikv_last_error().decode()
    assert lib.minikv_paged_decode_fp8_workspace_bytes(2, 8, 4, 80, 10, 16, 4, _lib.BF16) == -1
    rc = lib.minikv_kv_scatter_slots_fp8(p, p, p, p, p, 4, 8, 4, 3, 5, 15, 15, 0.1, 0.1, 1, _lib.F16, None)
    assert rc == _lib.EINVAL and "multiple of 16" in lib.minikv_last_error().decode()
    rc = lib.minikv_kv_scatter_slots_fp8(p, p, p, p, p, 4, 8, 4, 2, 64, 128, 128, float("inf"), 0.1, 0, _lib.F16, None)
    assert rc == _lib.EINVAL and "scales" in lib.minikv_last_error().decode()
    rc = lib.minikv_kv_scatter_slots_fp8(p, p, p, p, p, 4, 8, 4, 2, 64, 128, 128, 0.1, 0.1, 2, _lib.F16, None)
    assert rc == _lib.EINVAL and "E4M3 or E5M2" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode_fp8(p, p, p, p, p, p, p, 1 << 20, 2, 8, 4, 128, 10, 16, 4, 0.1, 0.1, 5, _lib.BF16, None)
    assert rc == _lib.EINVAL and "E4M3 or E5M2" in lib.minikv_last_error().decode()


def test_fp8_pool_and_wrappers_validate_arguments_on_the_host():
    from myvllm_mini_engine_b200.cache import FP8KVCachePool
    from myvllm_mini_engine_b200.kernels import paged_attention_fp8, write_kv_cache_slots_fp8

    with pytest.raises(ValueError, match="kv_format"):
        FP8KVCachePool(1, 4, 16, 2, 64, k_scale=0.1, v_scale=0.1, kv_format="e3m4", device="cpu")
    with pytest.raises(ValueError, match="finite and positive"):
        FP8KVCachePool(1, 4, 16, 2, 64, k_scale=0.0, v_scale=0.1, device="cpu")
    with pytest.raises(ValueError, match="even head_dim"):
        FP8KVCachePool(1, 4, 16, 2, 63, k_scale=0.1, v_scale=0.1, device="cpu")
    pool = FP8KVCachePool(2, 4, 16, 2, 64, k_scale=0.1, v_scale=0.1, kv_format="e5m2", device="cpu")
    assert pool.memory_bytes == 2 * 2 * 4 * 16 * 2 * 64 and pool.key.dtype == torch.uint8
    rows = torch.zeros(3, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(IndexError, match="layer"):
        pool.write_range(2, [0], 0, rows, rows)
    with pytest.raises(IndexError, match="block id"):
        pool.write_range(0, [7], 0, rows, rows)
    with pytest.raises(ValueError, match="capacity"):
        pool.write_range(0, [0], 15, rows, rows)
    with pytest.raises(ValueError, match="CUDA"):  # no CPU path
        pool.write_slots(0, torch.arange(3), rows, rows)
    kc = torch.zeros(4, 16, 2, 64, dtype=torch.uint8)
    with pytest.raises(ValueError, match="uint8 or a float8"):
        write_kv_cache_slots_fp8(kc.float(), kc.float(), torch.arange(3), rows, rows, 0.1, 0.1)
    with pytest.raises(ValueError, match="FP32/FP16/BF16"):
        write_kv_cache_slots_fp8(kc, kc.clone(), torch.arange(3), rows.to(torch.int32), rows.to(torch.int32), 0.1, 0.1)
    with pytest.raises(RuntimeError, match="CUDA"):
        paged_attention_fp8(torch.zeros(1, 4, 64, dtype=torch.bfloat16), kc, kc, torch.zeros(1, 1, dtype=torch.int64),
                            torch.ones(1, dtype=torch.int64), 16, 0.1, 0.1)


def test_fp8_pool_dtype_decides_the_format():
    from myvllm_mini_engine_b200.kernels import paged_attention_fp8, write_kv_cache_slots_fp8
    from myvllm_mini_engine_b200.kernels.fp8 import FORMATS, _format

    assert _format(None, torch.float8_e5m2) == FORMATS["e5m2"]
    assert _format("e4m3", torch.float8_e4m3fn) == FORMATS["e4m3"]
    assert _format(None) == FORMATS["e4m3"] and _format("e5m2", torch.uint8) == FORMATS["e5m2"]
    kc = torch.zeros(4, 16, 2, 64, dtype=torch.float8_e5m2)
    rows = torch.zeros(3, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="contradicts"):  # an e5m2 pool read as e4m3 would decode wrong values
        write_kv_cache_slots_fp8(kc, kc.clone(), torch.arange(3), rows, rows, 0.1, 0.1, kv_format="e4m3")
    with pytest.raises(ValueError, match="contradicts"):
        paged_attention_fp8(torch.zeros(1, 4, 64, dtype=torch.bfloat16), kc, kc, torch.zeros(1, 1, dtype=torch.int64),
                            torch.ones(1, dtype=torch.int64), 16, 0.1, 0.1, kv_format="e4m3")


def test_fp16_placements_of_fp8_codes_are_exact():
    """The bit placements the kernels use to turn codes into fp16 operands, restated in numpy
    and checked on every finite code against the oracle's decoder: an E5M2 code is the high
    byte of the fp16 of its value; an E4M3 code shifted down one bit inside the high byte, with
    its sign moved back to bit 15, is the fp16 of 2^-8 times its value (subnormals included)."""
    codes = np.arange(256, dtype=np.uint32)
    e5m2 = (codes << 8).astype(np.uint16).view(np.float16).astype(np.float64)
    ref5 = fp8_kv.decode_fp8(codes.astype(np.uint8), "e5m2").astype(np.float64)
    finite5 = np.isfinite(ref5)
    assert np.array_equal(e5m2[finite5], ref5[finite5])
    t = (codes << 8) >> 1
    e4m3 = ((t + (t & 0x4000)) & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float64)
    ref4 = fp8_kv.decode_fp8(codes.astype(np.uint8), "e4m3").astype(np.float64)
    finite4 = np.isfinite(ref4)
    assert finite4.sum() == 254  # 0x7f and 0xff are NaN
    assert np.array_equal(e4m3[finite4] * 256.0, ref4[finite4])
