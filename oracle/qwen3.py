"""Oracle: one batched Qwen3 decode step.  Test infrastructure only (see oracle/__init__).

Restates ``NativeQwen3.forward_decode_batch`` of the reference
(``mini_engine/model/native_qwen3.py:423-456``) with every backend set to
"torch" and the projections fused (``enable_projection_fusion``,
native_qwen3.py:362-376; ``FusedLinear`` computes ``torch.mm(x, W.t())``,
``kernels/linear.py:116-130``):

  * embedding        ``F.embedding``                    (data.py:14-19)
  * rotary tables    inv_freq / angles / cos, sin        (native_qwen3.py:449-452)
  * per layer        ``DecoderLayer.forward_decode_batch`` (native_qwen3.py:272-280)
      - input RMSNorm                                     (fallback.py:8-10)
      - q|k|v = mm(h, Wqkv^T), split, contiguous          (native_qwen3.py:99-112)
      - q_norm / k_norm, apply_rope                       (native_qwen3.py:175-182; fallback.py:13-20)
      - write_kv_cache_batch (torch path: one row per request, data.py:67-81)
      - paged_attention over lengths = positions + 1     (fallback.py:27-64, via oracle.paged_decode)
      - o_proj, residual_rms_norm, gate|up mm, silu_and_mul, down, residual_add
                                                          (native_qwen3.py:232-240, 272-280; elementwise.py)
  * final RMSNorm and the tied LM head ``mm(x, E^T)``     (native_qwen3.py:456)

The functions are plain torch and run wherever their tensors live: on the CPU
for the golden pin against the reference, and on the GPU under test as the
eager reference model run "with torch backends on the same GPU and the same
KV state", which is how the reference validates its own model paths.
``weights`` is any object with the attributes of
``myvllm_mini_engine_b200.engine.qwen3.Qwen3Weights`` (embed, norm, layers[i].
{input_norm, qkv, q_norm, k_norm, o, post_norm, gate_up, down}).
"""

from __future__ import annotations

import torch
from torch.nn import functional as F

from . import paged_decode


def rms_norm(x, weight, eps):
    """fallback.py:8-10."""
    variance = x.float().pow(2).mean(dim=-1, keepdim=True)
    return (x.float() * torch.rsqrt(variance + eps)).to(x.dtype) * weight


def apply_rope(q, k, cos, sin):
    """fallback.py:13-20 (cos/sin broadcast over heads)."""
    half = q.shape[-1] // 2
    q1, q2 = q[..., :half], q[..., half:]
    k1, k2 = k[..., :half], k[..., half:]
    q_out = torch.cat((q1 * cos - q2 * sin, q1 * sin + q2 * cos), dim=-1)
    k_out = torch.cat((k1 * cos - k2 * sin, k1 * sin + k2 * cos), dim=-1)
    return q_out, k_out


def silu_and_mul(gate, up):
    """fallback.py:23-24."""
    return F.silu(gate) * up


def rope_tables(positions, head_dim, theta, dtype):
    """native_qwen3.py:449-452."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=positions.device).float() / head_dim))
    angles = positions.to(dtype=torch.float32)[:, None] * inv_freq[None, :]
    return angles.cos().to(dtype), angles.sin().to(dtype)


def append_rows(key_cache, value_cache, block_tables, positions, key, value, block_size):
    """write_kv_cache_batch, torch path (data.py:76-79 -> data.py:51-62), one token per request."""
    tables = block_tables.cpu()
    for batch, position in enumerate(positions.cpu().tolist()):
        page = int(tables[batch, position // block_size])
        key_cache[page, position % block_size] = key[batch]
        value_cache[page, position % block_size] = value[batch]


def decode_step(config, weights, input_ids, key_pool, value_pool, block_tables, positions, attention=None):
    """Logits ``[B, vocab]`` of one decode step; appends each request's K/V to the pools.

    ``key_pool``/``value_pool`` are ``[layers, num_blocks, block_size, kv_heads,
    head_dim]`` and are modified in place, like the reference's KVCachePool.
    ``attention`` replaces the decode attention (default: the reference's,
    ``paged_decode.paged_attention``) -- for test controls only.
    """
    attention = paged_decode.paged_attention if attention is None else attention
    cfg = config
    hq, hkv, dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    block_size = key_pool.shape[2]
    batch = input_ids.shape[0]
    x = F.embedding(input_ids, weights.embed)
    cos, sin = rope_tables(positions, dim, cfg.rope_theta, x.dtype)
    lengths = positions + 1
    for layer, w in enumerate(weights.layers):
        h = rms_norm(x, w.input_norm, cfg.rms_norm_eps)
        qkv = torch.mm(h, w.qkv.t())
        q_raw, k_raw, v_raw = qkv.split((hq * dim, hkv * dim, hkv * dim), dim=-1)
        q = q_raw.contiguous().view(batch, hq, dim)
        k = k_raw.contiguous().view(batch, hkv, dim)
        v = v_raw.contiguous().view(batch, hkv, dim)
        q = rms_norm(q, w.q_norm, cfg.rms_norm_eps)
        k = rms_norm(k, w.k_norm, cfg.rms_norm_eps)
        q, k = apply_rope(q, k, cos.unsqueeze(1), sin.unsqueeze(1))
        append_rows(key_pool[layer], value_pool[layer], block_tables, positions, k, v, block_size)
        attended = attention(q, key_pool[layer], value_pool[layer], block_tables, lengths, block_size)
        o = torch.mm(attended.reshape(batch, -1), w.o.t())
        summed = o + x
        normalized = rms_norm(summed, w.post_norm, cfg.rms_norm_eps)
        gate, up = (part.contiguous() for part in torch.mm(normalized, w.gate_up.t()).chunk(2, dim=-1))
        x = summed + torch.mm(silu_and_mul(gate, up), w.down.t())
    return torch.mm(rms_norm(x, weights.norm, cfg.rms_norm_eps), weights.lm_head.t())


def top2_margin(logits):
    """Gap between the largest and second-largest logit of each row (fp32)."""
    top = torch.topk(logits.float(), 2, dim=-1).values
    return top[:, 0] - top[:, 1]
