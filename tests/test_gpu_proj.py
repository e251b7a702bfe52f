"""Fused tcgen05 projections of the decode step (csrc/proj.cu) on the GPU.

Checkers:
  * the projection itself (``minikv_linear``) against the float64 product of
    the same 16-bit operands: every output within half a unit in the last
    place of the exact value plus the fp32 accumulation bound
    (2^-20 * sum_k |x_k w_k|, which matters only where the sum cancels), and
    bit-exact on integer operands whose sums are exact in every precision;
  * every fused prologue / epilogue against the reference's op chain
    (``oracle.qwen3`` rms_norm, silu_and_mul, apply_rope, append_rows, and the
    residual add) applied to the plain projection of the same kernel: the
    split over in-features depends only on the shapes, so the fused and the
    plain launch accumulate identically and the chain must match bit for bit;
  * determinism: two launches give identical bits.
"""

import pytest
import torch

import cases
from myvllm_mini_engine_b200 import _lib
from myvllm_mini_engine_b200.engine.qwen3 import pack_linear
from oracle import qwen3 as ref

pytestmark = pytest.mark.gpu


def stream():
    return torch.cuda.current_stream().cuda_stream


def ulps(a, b):
    def ordered(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -32768 - i, i)
    return (ordered(a) - ordered(b)).abs()


def rand(gen, *shape, dtype, scale=1.0):
    return (scale * torch.randn(*shape, device="cuda", generator=gen)).to(dtype)


def linear(x, w, ss=None, norm=None, eps=1e-6):
    out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device="cuda")
    _lib.check(_lib.load().minikv_linear(x.data_ptr(), x.stride(0), None if ss is None else ss.data_ptr(),
                                         None if norm is None else norm.data_ptr(), eps, pack_linear(w).data_ptr(),
                                         out.data_ptr(), x.shape[0], x.shape[1], w.shape[0],
                                         _lib.dtype_code(x.dtype), stream()), "linear")
    return out


def unpack(packed, rows, cols, pair_offset=0):
    """Row-major weight back from the packed layout (torch restatement of the layout)."""
    blocks = packed.view(-1, cols // 64, 128, 8, 8)  # [tile, k-block, row, chunk, element]
    r = torch.arange(128, device=packed.device)
    logical = torch.arange(8, device=packed.device)[None, :] ^ (r[:, None] % 8)  # chunk holding logical chunk
    gathered = blocks[:, :, r[:, None], logical]  # [tile, kb, row, logical chunk, element]
    tiles = gathered.permute(0, 2, 1, 3, 4).reshape(-1, 128, cols)
    if pair_offset == 0:
        return tiles.reshape(rows, cols)
    return torch.cat([tiles[:, :64].reshape(-1, cols), tiles[:, 64:].reshape(-1, cols)])


@pytest.mark.parametrize("rows,cols,pair", [(128, 64, 0), (4096, 1024, 0), (6144, 1024, 3072), (256, 192, 128)])
def test_pack_linear_layout(cuda_device, rows, cols, pair):
    gen = torch.Generator(device="cuda").manual_seed(rows + cols)
    w = torch.randn(rows, cols, device="cuda", generator=gen).to(torch.bfloat16)
    packed = pack_linear(w, pair_offset=pair)
    assert torch.equal(unpack(packed, rows, cols, pair), w)


def tile_sums(x):
    """Per-row sums of squares over 128-feature tiles, [features / 128, rows] fp32 (rounded values)."""
    xf = x.float()
    return (xf * xf).view(x.shape[0], -1, 128).sum(-1).t().contiguous()


def normalised(x, ss, weight, eps):
    """T(T(x * rsqrt(ss / n + eps)) * w) with the partial sums added in tile order, as the prologue does."""
    total = ss[0].clone()
    for j in range(1, ss.shape[0]):
        total = total + ss[j]
    inv = torch.rsqrt(total / x.shape[1] + eps)
    return ((x.float() * inv[:, None]).to(x.dtype).float() * weight.float()).to(x.dtype)


SHAPES = [  # tokens, in_features, out_features
    (1, 1024, 4096), (7, 64, 128), (16, 2048, 1024), (32, 1024, 4096), (32, 3072, 1024),
    (33, 1024, 1024), (100, 1024, 6144), (256, 1024, 4096), (300, 2048, 1024),
]


def spacing(y, dtype):
    """Distance between neighbouring ``dtype`` values at |y| (normal range; fp16 subnormals included)."""
    mant, low = (7, -133) if dtype == torch.bfloat16 else (10, -14)
    e = torch.floor(torch.log2(y.abs().clamp_min(1e-300)))
    return torch.exp2(torch.clamp(e, min=low) - mant)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens,k,n", SHAPES)
def test_linear_matches_exact_projection(cuda_device, dtype, tokens, k, n):
    gen = torch.Generator(device="cuda").manual_seed(tokens * 7 + k + n)
    x = rand(gen, tokens, k, dtype=dtype)
    w = rand(gen, n, k, dtype=dtype, scale=0.02)
    out = linear(x, w)
    exact = x.double() @ w.double().t()
    bound = 0.5 * spacing(exact, dtype) + 2.0 ** -20 * (x.double().abs() @ w.double().abs().t())
    assert ((out.double() - exact).abs() <= bound).all()
    assert torch.equal(out, linear(x, w))  # deterministic
    # operands in {-1, 0, 1}: every partial sum is an exact small integer
    xi = torch.randint(-1, 2, (tokens, k), device="cuda", generator=gen).to(dtype)
    wi = torch.randint(-1, 2, (n, k), device="cuda", generator=gen).to(dtype)
    assert torch.equal(linear(xi, wi), (xi.double() @ wi.double().t()).to(dtype))
    assert _lib.device_status() == 0


def test_linear_reads_strided_rows(cuda_device):
    gen = torch.Generator(device="cuda").manual_seed(3)
    big = rand(gen, 40, 1024 + 64, dtype=torch.bfloat16)
    x = big[:, 64:]  # row stride 1088 elements, base 128 bytes in
    w = rand(gen, 256, 1024, dtype=torch.bfloat16, scale=0.02)
    assert torch.equal(linear(x, w), linear(x.contiguous(), w))


@pytest.mark.parametrize("tokens", [5, 32, 256])
def test_rms_norm_prologue(cuda_device, tokens):
    dtype, k, eps = torch.bfloat16, 1024, 1e-6
    gen = torch.Generator(device="cuda").manual_seed(tokens)
    x = rand(gen, tokens, k, dtype=dtype, scale=3.0)
    norm = (1 + 0.1 * torch.randn(k, device="cuda", generator=gen)).to(dtype)
    w = rand(gen, 2048, k, dtype=dtype, scale=0.02)
    ss = tile_sums(x)
    fused = linear(x, w, ss, norm, eps)
    assert torch.equal(fused, linear(normalised(x, ss, norm, eps), w))
    # and the reference's RMSNorm (its own reduction order) within one ulp before the projection
    expected = (ref.rms_norm(x, norm, eps).float() @ w.float().t()).to(dtype)
    torch.testing.assert_close(fused.float(), expected.float(), atol=0.02, rtol=0.02)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens,k,n", [(1, 2048, 1024), (32, 2048, 1024), (32, 3072, 1024), (200, 1024, 512)])
def test_linear_residual(cuda_device, dtype, tokens, k, n):
    gen = torch.Generator(device="cuda").manual_seed(11 + tokens)
    x = rand(gen, tokens, k, dtype=dtype)
    w = rand(gen, n, k, dtype=dtype, scale=0.02)
    residual = rand(gen, tokens, n, dtype=dtype)
    out = torch.empty_like(residual)
    ss = torch.full((n // 128, tokens), float("nan"), device="cuda")
    _lib.check(_lib.load().minikv_linear_residual(x.data_ptr(), k, pack_linear(w).data_ptr(), residual.data_ptr(),
                                                  out.data_ptr(),
                                                  ss.data_ptr(), tokens, k, n, _lib.dtype_code(dtype), stream()),
               "linear_residual")
    expected = linear(x, w) + residual  # torch's 16-bit add: fp32 sum rounded once
    assert torch.equal(out, expected)
    torch.testing.assert_close(ss, tile_sums(out), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tokens", [3, 32, 129])
def test_linear_silu_mul(cuda_device, tokens):
    dtype, k, inter, eps = torch.bfloat16, 1024, 3072, 1e-6
    gen = torch.Generator(device="cuda").manual_seed(21 + tokens)
    x = rand(gen, tokens, k, dtype=dtype)
    norm = (1 + 0.1 * torch.randn(k, device="cuda", generator=gen)).to(dtype)
    w = rand(gen, 2 * inter, k, dtype=dtype, scale=0.05)
    lib = _lib.load()
    for ss in (None, tile_sums(x)):
        out = torch.empty(tokens, inter, dtype=dtype, device="cuda")
        _lib.check(lib.minikv_linear_silu_mul(x.data_ptr(), k, None if ss is None else ss.data_ptr(),
                                              norm.data_ptr(), eps, pack_linear(w, pair_offset=inter).data_ptr(),
                                              out.data_ptr(), tokens, k, inter,
                                              _lib.BF16, stream()), "linear_silu_mul")
        source = x if ss is None else normalised(x, ss, norm, eps)
        gate_up = linear(source, w)
        expected = ref.silu_and_mul(gate_up[:, :inter].contiguous(), gate_up[:, inter:].contiguous())
        assert torch.equal(out, expected)


def test_linear_qk_rope_append(cuda_device):
    dtype, hq, hkv, dim, bs, k, eps = torch.bfloat16, 16, 8, 128, 16, 1024, 1e-6
    from myvllm_mini_engine_b200.engine.qwen3 import Qwen3Config

    cfg = Qwen3Config(vocab_size=64, hidden_size=k, intermediate_size=256, num_hidden_layers=1,
                      num_attention_heads=hq, num_key_value_heads=hkv, head_dim=dim)
    # contexts at page boundaries, an empty one, and one past its table (its rows are skipped)
    c = cases.qwen3_decode_case(cfg, dtype, contexts=(0, 15, 16, 300, 77, 31), block_size=bs, seed=12)
    batch = len(c["positions"])
    positions, tables = c["positions"].cuda(), c["block_tables"].cuda()
    positions[5] = tables.shape[1] * bs  # beyond the table: no append
    gen = torch.Generator(device="cuda").manual_seed(13)
    x = rand(gen, batch, k, dtype=dtype, scale=2.0)
    norm = (1 + 0.1 * torch.randn(k, device="cuda", generator=gen)).to(dtype)
    w = rand(gen, (hq + 2 * hkv) * dim, k, dtype=dtype, scale=0.05)
    qw = (1 + 0.1 * torch.randn(dim, device="cuda", generator=gen)).to(dtype)
    kw = (1 + 0.1 * torch.randn(dim, device="cuda", generator=gen)).to(dtype)
    cos, sin = ref.rope_tables(positions, dim, cfg.rope_theta, dtype)
    kc0, vc0 = c["key_pool"][0].cuda(), c["value_pool"][0].cuda()
    lib = _lib.load()
    for ss in (None, tile_sums(x)):
        kc, vc = kc0.clone(), vc0.clone()
        q = torch.empty(batch, hq, dim, dtype=dtype, device="cuda")
        _lib.check(lib.minikv_linear_qk_rope_append(
            x.data_ptr(), k, None if ss is None else ss.data_ptr(), norm.data_ptr(), eps, pack_linear(w).data_ptr(),
            qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
            tables.data_ptr(), positions.data_ptr(), batch, k, hq, hkv, dim, kc.shape[0], bs, tables.shape[1],
            _lib.BF16, stream()), "linear_qk_rope_append")
        # the chain: plain projection, then the standalone q/k-norm + RoPE + append kernel
        qkv = linear(x if ss is None else normalised(x, ss, norm, eps), w)
        kc_ref, vc_ref = kc0.clone(), vc0.clone()
        q_ref = torch.empty_like(q)
        _lib.check(lib.minikv_qk_rope_append(qkv.data_ptr(), qkv.stride(0), qw.data_ptr(), kw.data_ptr(),
                                             cos.data_ptr(), sin.data_ptr(), q_ref.data_ptr(), kc_ref.data_ptr(),
                                             vc_ref.data_ptr(), tables.data_ptr(), positions.data_ptr(), batch, hq,
                                             hkv, dim, kc.shape[0], bs, tables.shape[1], eps, _lib.BF16, stream()),
                   "qk_rope_append")
        assert torch.equal(q, q_ref)
        assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)
        assert not torch.equal(kc, kc0)  # rows were appended
    assert _lib.device_status() == 0


def test_projection_shape_errors(cuda_device):
    lib = _lib.load()
    x = torch.zeros(4, 96, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(128, 96, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    rc = lib.minikv_linear(x.data_ptr(), 96, None, None, 1e-6, w.data_ptr(), out.data_ptr(), 4, 96, 128, _lib.BF16,
                           stream())
    assert rc == _lib.EINVAL and "multiple of 64" in lib.minikv_last_error().decode()
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(96, 128, dtype=torch.bfloat16, device="cuda")
    rc = lib.minikv_linear(x.data_ptr(), 128, None, None, 1e-6, w.data_ptr(), out.data_ptr(), 4, 128, 96, _lib.BF16,
                           stream())
    assert rc == _lib.EINVAL and "multiple of 128" in lib.minikv_last_error().decode()
