"""CPU oracle: the FP8 (E4M3 / E5M2) KV pool.  Test infrastructure only (see oracle/__init__).

The reference has no FP8 KV pool; it lists one as future work
(``VALIDATION_AND_BENCHMARKS.md:375``).  Its contract here is therefore ours,
and its parity is pinned against torch's own ``float8_e4m3fn`` conversion
and ``float8_e5m2`` conversions (tests/test_fp8_oracle_cpu.py), not against
reference outputs:

* storage: one byte per element, OCP FP8 E4M3 ("e4m3fn": 1 sign bit, 4
  exponent bits with bias 7, 3 mantissa bits, no infinities, S.1111.111 is
  NaN, largest finite 448) or E5M2 (5 exponent bits with bias 15, 2 mantissa
  bits, IEEE-style infinities and NaNs, largest finite 57344), in a pool shaped
  like the 16-bit one, ``[num_blocks, block_size, kv_heads, head_dim]``;
* one fp32 scale for keys and one for values: ``stored = fp8(x * (1/scale))``
  with the product rounded to fp32 first, then rounded to nearest-even and
  saturated to the largest finite value (infinities too); NaN becomes 0x7F;
* attention reads ``stored * scale``: the oracle dequantises the pool to fp32
  and runs the trusted-mode decode oracle (oracle/paged_decode.py), which
  restates ``mini_engine/kernels/fallback.py:27-64`` with the CUDA kernel's
  guards (``csrc/paged_attention.cu:62-83, 99-121``);
* the slot scatter follows ``write_kv_cache_slots`` (``data.py:84-130``,
  ``csrc/data.cu:196-206``): a slot outside the capacity writes nothing.
"""

from __future__ import annotations

import numpy as np
import torch

from .paged_decode import paged_attention_trusted_fp32

E4M3_MAX = 448.0
E5M2_MAX = 57344.0
# format -> (exponent bits, mantissa bits, bias, largest finite value)
FORMATS = {"e4m3": (4, 3, 7, E4M3_MAX), "e5m2": (5, 2, 15, E5M2_MAX)}


def encode_fp8(x, fmt="e4m3") -> np.ndarray:
    """Round float32 values to OCP FP8 codes (uint8): nearest-even, saturating to the largest finite value."""
    ebits, mbits, bias, vmax = FORMATS[fmt]
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    x = x.reshape(-1)
    nan = np.isnan(x)
    a = np.abs(np.where(nan, np.float32(0), x).astype(np.float64))
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.minimum(a, vmax)  # saturate (an infinity too) before rounding
    code = np.zeros(x.shape, dtype=np.int64)
    normal = a >= 2.0 ** (1 - bias)
    # subnormal range: multiples of 2^(1-bias-mbits); rounding up to the smallest
    # normal gives code 2^mbits (exponent field 1, mantissa 0), which is right
    code[~normal] = np.rint(a[~normal] * 2.0 ** (bias - 1 + mbits)).astype(np.int64)
    if normal.any():
        an = a[normal]
        _, e2 = np.frexp(an)            # an = f * 2^e2, f in [0.5, 1)
        e = e2.astype(np.int64) - 1     # an in [2^e, 2^(e+1))
        steps = np.rint(an / np.exp2(e - mbits)).astype(np.int64)  # in [2^m, 2^(m+1)], exact scaling
        carry = steps == 2 ** (mbits + 1)
        e = np.where(carry, e + 1, e)
        steps = np.where(carry, 2 ** mbits, steps)
        code[normal] = ((e + bias) << mbits) | (steps - 2 ** mbits)
    out = (code.astype(np.uint8) | sign).astype(np.uint8)
    out[nan] = 0x7F
    return out.reshape(shape)


def encode_e4m3(x) -> np.ndarray:
    """Round float32 values to E4M3 codes (uint8): nearest-even, saturating."""
    return encode_fp8(x, "e4m3")


def _table(fmt) -> np.ndarray:
    ebits, mbits, bias, _ = FORMATS[fmt]
    codes = np.arange(256)
    mag = codes & 0x7F
    exp = mag >> mbits
    man = mag & ((1 << mbits) - 1)
    value = np.where(exp == 0, man * 2.0 ** (1 - bias - mbits), (1.0 + man / 2.0 ** mbits) * np.exp2(exp - bias * 1.0))
    top = (1 << ebits) - 1
    if fmt == "e4m3":
        value[mag == 0x7F] = np.nan            # S.1111.111 is NaN, no infinities
    else:
        value[(exp == top) & (man == 0)] = np.inf   # IEEE-style: infinities and NaNs
        value[(exp == top) & (man != 0)] = np.nan
    value = np.where(codes & 0x80, -value, value)
    return value.astype(np.float32)


DECODE_TABLES = {fmt: _table(fmt) for fmt in FORMATS}
DECODE_TABLE = DECODE_TABLES["e4m3"]


def decode_fp8(codes, fmt="e4m3") -> np.ndarray:
    """float32 values of FP8 codes."""
    return DECODE_TABLES[fmt][np.asarray(codes, dtype=np.uint8).astype(np.int64)]


def decode_e4m3(codes) -> np.ndarray:
    """float32 values of E4M3 codes."""
    return decode_fp8(codes, "e4m3")


def quantize(x: torch.Tensor, scale: float, fmt: str = "e4m3") -> np.ndarray:
    """Codes of ``x * (1/scale)``: the product rounded to fp32, then to the FP8 format."""
    inv = np.float32(1.0) / np.float32(scale)
    prod = (x.detach().float().cpu().numpy() * inv).astype(np.float32)
    return encode_fp8(prod, fmt)


def dequantize(codes: torch.Tensor, scale: float, fmt: str = "e4m3") -> torch.Tensor:
    """fp32 tensor ``decode(codes) * scale`` (the values attention reads)."""
    values = decode_fp8(codes.cpu().numpy(), fmt) * np.float32(scale)
    return torch.from_numpy(values.astype(np.float32))


def scatter_slots_fp8(key_cache, value_cache, slot_mapping, key, value, k_scale, v_scale, fmt="e4m3"):
    """``rows[slot_mapping[t]] = quantize(key[t])`` (and value), in place on uint8 CPU pools.

    ``key``/``value`` are ``[tokens, kv_heads, head_dim]`` (any float dtype),
    the pools ``[num_blocks, block_size, kv_heads, head_dim]`` uint8.
    """
    kc = key_cache.numpy().reshape(-1, key_cache.shape[2] * key_cache.shape[3])
    vc = value_cache.numpy().reshape(-1, value_cache.shape[2] * value_cache.shape[3])
    kq = quantize(key, k_scale, fmt).reshape(key.shape[0], -1)
    vq = quantize(value, v_scale, fmt).reshape(value.shape[0], -1)
    capacity = kc.shape[0]
    for t, slot in enumerate(slot_mapping.cpu().tolist()):
        if 0 <= slot < capacity:  # data.cu:196-206
            kc[slot] = kq[t]
            vc[slot] = vq[t]


def paged_attention_fp8_fp32(query, key_cache, value_cache, block_tables, context_lens, block_size,
                             k_scale, v_scale, fmt="e4m3"):
    """fp32 decode attention over an FP8 pool, read as ``code * scale``."""
    keys = dequantize(key_cache, k_scale, fmt)
    values = dequantize(value_cache, v_scale, fmt)
    return paged_attention_trusted_fp32(query.float().cpu(), keys, values, block_tables, context_lens,
                                        block_size)
