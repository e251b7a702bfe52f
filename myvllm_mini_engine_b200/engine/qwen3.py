"""Batched Qwen3 decode step over the paged KV pool.

The caller of the paged-KV path in the reference engine is
``NativeQwen3.forward_decode_batch`` (``mini_engine/model/native_qwen3.py:423-456``):
per layer it runs RMSNorm, the q|k|v projection, q/k RMSNorm + RoPE, the
decode KV append, paged decode attention, the output projection and the MLP.
This module runs the same step on B200 with the sm_100a kernels of libminikv.
By default (``fused_projections``, head_dim 128) a batch of at most
``FUSED_MAX_BATCH`` requests runs every projection on the tcgen05 projection
kernels (packed weights) with the element-wise steps fused into them:

    per layer (5 launches):  q|k|v projection [RMSNorm prologue; q/k RMSNorm +
                             RoPE epilogue, new K/V to staging rows] | KV append
                             + paged decode | o projection [+ residual] |
                             gate|up projection [RMSNorm prologue; SiLU * up] |
                             down projection [+ residual]

where each residual epilogue hands the next RMSNorm its per-row sums of
squares, and each projection streams its weights while the previous kernel
finishes (chained launches).  Larger batches, and ``fused_projections=False``,
run the projections as plain cuBLAS GEMMs through ``torch.mm`` (the reference's
``FusedLinear`` torch path, ``kernels/linear.py:116-130``) around the fused
element-wise kernels:

    per layer (9 launches):  RMSNorm | mm(q|k|v) | qk-norm + RoPE (new K/V to
                             staging rows) | KV append + paged decode | mm(o) |
                             residual + RMSNorm | mm(gate|up) | SiLU * up | mm(down)

with the residual add of the MLP fused into the next layer's RMSNorm.  The
decode is ``paged_attention_with_append``, chained: the kernel before it writes
only q and the staging rows, so the decode starts staging pool rows while that
kernel finishes, and writes the staged rows into the pool itself.  That
composition reproduces the reference's rounding bit for bit except inside
the decode attention.  Either way rounding follows the eager reference
(every intermediate in the model dtype), so the step's greedy tokens match
the reference model's on the same weights and KV state.  The step never
synchronises with the host, so it can be captured in a CUDA graph
(:class:`DecodeGraph`).

Weights use the fused layouts of ``enable_projection_fusion``
(native_qwen3.py:362-376): ``qkv = cat(Wq, Wk, Wv)`` and ``gate_up = cat(Wg, Wu)``,
each ``[out_features, in_features]`` like ``nn.Linear``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch.nn import functional as F

from .. import _lib
from ..cache.kv_cache import FP8KVCachePool, PagedKVPool
from ..kernels.fp8 import paged_attention_fp8_with_append
from ..kernels.paged import paged_attention_with_append


@dataclass(frozen=True)
class Qwen3Config:
    """Dense Qwen3 architecture (fields of ``Qwen3Config``, native_qwen3.py:21-42)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position_embeddings: int = 32768
    attention_bias: bool = False
    tie_word_embeddings: bool = True

    def __post_init__(self):
        for name in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                     "num_attention_heads", "num_key_value_heads", "head_dim", "max_position_embeddings"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.num_attention_heads % self.num_key_value_heads or self.head_dim % 2:
            raise ValueError("Qwen3 requires divisible GQA heads and an even head_dim")
        if self.attention_bias:
            raise ValueError("attention bias is not supported by the decode step")

    @classmethod
    def qwen3_0_6b(cls, **overrides):
        """Qwen3-0.6B: 28 layers, hidden 1024, 16/8 heads of 128, SwiGLU 3072, vocab 151936, tied."""
        values = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
                      rope_theta=1000000.0, max_position_embeddings=40960, tie_word_embeddings=True)
        values.update(overrides)
        return cls(**values)


@dataclass
class LayerWeights:
    input_norm: torch.Tensor   # [H]
    qkv: torch.Tensor          # [(Hq + 2 Hkv) D, H]
    q_norm: torch.Tensor       # [D]
    k_norm: torch.Tensor       # [D]
    o: torch.Tensor            # [H, Hq D]
    post_norm: torch.Tensor    # [H]
    gate_up: torch.Tensor      # [2 I, H]
    down: torch.Tensor         # [H, I]


@dataclass
class Qwen3Weights:
    embed: torch.Tensor                      # [V, H]
    norm: torch.Tensor                       # [H]
    layers: list = field(default_factory=list)
    lm_head_weight: torch.Tensor | None = None  # [V, H]; None when tied to embed

    @property
    def lm_head(self) -> torch.Tensor:
        return self.embed if self.lm_head_weight is None else self.lm_head_weight

    @classmethod
    def random(cls, config: Qwen3Config, *, dtype=torch.bfloat16, device="cuda", seed=0, std=0.02):
        """Seeded random init: every projection and the embedding ~ N(0, std), norms = 1.

        Draw order (one ``torch.Generator`` on ``device``): embed, then per layer
        qkv, o, gate_up, down, then the untied LM head if any.  Each tensor is
        drawn in fp32 and rounded to ``dtype``.
        """
        cfg, device = config, torch.device(device)
        gen = torch.Generator(device=device).manual_seed(seed)

        def normal(*shape):
            return torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, std, generator=gen).to(dtype)

        def ones(n):
            return torch.ones(n, dtype=dtype, device=device)

        h, d, i = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
        qkv_rows = (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * d
        embed = normal(cfg.vocab_size, h)
        layers = []
        for _ in range(cfg.num_hidden_layers):
            qkv, o = normal(qkv_rows, h), normal(h, cfg.num_attention_heads * d)
            gate_up, down = normal(2 * i, h), normal(h, i)
            layers.append(LayerWeights(ones(h), qkv, ones(d), ones(d), o, ones(h), gate_up, down))
        head = None if cfg.tie_word_embeddings else normal(cfg.vocab_size, h)
        return cls(embed, ones(h), layers, head)


def _check(status, what):
    _lib.check(status, what)


_ARGMAX_WORKSPACES: dict = {}
_ARGMAX_RETIRED: list = []


def greedy_ids(logits: torch.Tensor) -> torch.Tensor:
    """Greedy next token of every row of ``logits [batch, vocab]``: ``logits.argmax(dim=-1)``.

    The reference samples greedily with ``logits.argmax(dim=-1)`` (``mini_engine/sampling.py:14-22``):
    a NaN counts as the largest value and ties take the lowest index.  ``minikv_argmax_rows``
    computes the same in two chained launches.  Its scratch (one key per warp of a row's column
    slices) is a buffer kept per CUDA stream (never freed, since a captured graph may use it).
    """
    if logits.ndim != 2 or not logits.is_cuda or logits.stride(1) != 1:
        raise ValueError("logits must be a 2D CUDA tensor with contiguous rows")
    lib = _lib.load()
    rows, cols = logits.shape
    need = lib.minikv_argmax_workspace_bytes(rows, cols)
    if need < 0:
        raise ValueError("argmax takes 1..65535 rows of at least one column")
    device = logits.device
    with _lib.on_device(device):
        stream = _lib.stream_of(device)
        key = (device.index, stream)
        ws = _ARGMAX_WORKSPACES.get(key)
        if ws is None or ws.numel() < need:
            if ws is not None:
                _ARGMAX_RETIRED.append(ws)
            ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
            _ARGMAX_WORKSPACES[key] = ws
        out = torch.empty(rows, dtype=torch.long, device=device)
        _check(lib.minikv_argmax_rows(logits.data_ptr(), rows, cols, logits.stride(0), _lib.dtype_code(logits.dtype),
                                      ws.data_ptr(), ws.numel(), out.data_ptr(), stream), "argmax_rows")
    return out


def pack_linear(weight: torch.Tensor, *, pair_offset: int = 0) -> torch.Tensor:
    """A packed copy of an ``[out_features, in_features]`` weight for the fused projections.

    The layout is the one ``minikv_pack_linear`` documents (``include/minikv.h``):
    blocks of 128 rows x 64 in-features, each stored as the tensor core reads it
    from shared memory.  ``pair_offset`` (the intermediate size) packs a fused
    gate|up weight so that each block row holds matching gate and up rows.
    """
    if weight.ndim != 2 or not weight.is_contiguous() or not weight.is_cuda:
        raise ValueError("pack_linear expects a contiguous 2D CUDA weight")
    packed = torch.empty_like(weight)
    with _lib.on_device(weight.device):
        _check(_lib.load().minikv_pack_linear(weight.data_ptr(), packed.data_ptr(), weight.shape[0], weight.shape[1],
                                              pair_offset, _lib.dtype_code(weight.dtype),
                                              torch.cuda.current_stream(weight.device).cuda_stream), "pack_linear")
    return packed


class Qwen3DecodeStep:
    """One decode token per request through all layers, reading and appending the paged pool.

    ``pool`` is a :class:`PagedKVPool` (or the reference engine's ``KVCachePool``) shaped for ``config`` (layers, kv heads,
    head_dim) in the weights' dtype and device, or an :class:`FP8KVCachePool`
    (an extension: the new token's K/V are written by the same kernels into a
    small bf16 staging buffer, then quantised into the pool by the FP8 slot
    scatter, and the attention reads the FP8 pool).  ``forward_decode_batch``
    follows ``NativeQwen3.forward_decode_batch`` (native_qwen3.py:423-456):
    it returns the logits ``[B, vocab]`` and appends each request's new K/V at
    ``positions[b]`` through ``block_tables[b]``.
    """

    #: batches up to this size take the fused tcgen05 projections; larger ones cuBLAS
    FUSED_MAX_BATCH = 32

    def __init__(self, config: Qwen3Config, weights: Qwen3Weights, pool: PagedKVPool, *,
                 fused_projections: bool | None = None):
        shape = pool.shape
        if (shape.num_layers, shape.num_kv_heads, shape.head_dim) != (
                config.num_hidden_layers, config.num_key_value_heads, config.head_dim):
            raise ValueError("KV cache architecture mismatch")
        self.fp8 = isinstance(pool, FP8KVCachePool)
        if pool.key.device != weights.embed.device or (not self.fp8 and pool.dtype != weights.embed.dtype):
            raise ValueError("cache must match model device and dtype")
        if weights.embed.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("the decode step runs in FP16/BF16")
        if config.head_dim not in (64, 128, 256):
            raise ValueError("the decode step supports head_dim 64, 128 or 256")
        self.config, self.weights, self.pool = config, weights, pool
        self.code = _lib.dtype_code(weights.embed.dtype)
        self.lib = _lib.load()
        fusable = self.fusable(config)
        if fused_projections and not fusable:
            raise ValueError("fused projections need head_dim 128, hidden and q-head sizes that are multiples "
                             "of 128 and an intermediate size that is a multiple of 64")
        self.fused_projections = fusable if fused_projections is None else bool(fused_projections)
        # Rotary tables of every position, computed once with the torch ops the reference applies per
        # step (inv_freq, fp32 angles, cos/sin rounded to the model dtype), so a step's rows are
        # bit-identical to computing them on the fly; a step gathers its rows.
        dim, device = config.head_dim, weights.embed.device
        inv_freq = 1.0 / (config.rope_theta ** (torch.arange(0, dim, 2, device=device).float() / dim))
        angles = torch.arange(config.max_position_embeddings, device=device, dtype=torch.float32)[:, None] * inv_freq
        self._cos_table = angles.cos().to(weights.embed.dtype)
        self._sin_table = angles.sin().to(weights.embed.dtype)
        del angles
        self._stage_index = {}
        self._packed = []
        if self.fused_projections:
            # the fused projections read packed weights (copies made once, here)
            inter = config.intermediate_size
            self._packed = [(pack_linear(layer.qkv), pack_linear(layer.o),
                             pack_linear(layer.gate_up, pair_offset=inter), pack_linear(layer.down))
                            for layer in weights.layers]

    @staticmethod
    def fusable(config: Qwen3Config) -> bool:
        """Shapes the fused tcgen05 projections take (Qwen3 models use head_dim 128)."""
        return (config.head_dim == 128 and config.hidden_size % 128 == 0
                and (config.num_attention_heads * config.head_dim) % 128 == 0
                and config.intermediate_size % 64 == 0)

    # ------------------------------------------------------------ fused ops
    def _rotary(self, positions):
        """cos / sin rows ``[batch, head_dim / 2]`` of the positions, gathered from the tables.

        Positions are clamped into the table (a captured graph skips the host range check; the
        KV kernels guard the pool on their own), so the gather never reads outside it.
        """
        rows = positions.clamp(0, self._cos_table.shape[0] - 1)
        return self._cos_table.index_select(0, rows), self._sin_table.index_select(0, rows)

    def _rms(self, x, residual, weight, out, sum_out, stream):
        _check(self.lib.minikv_rms_norm(x.data_ptr(), None if residual is None else residual.data_ptr(),
                                        weight.data_ptr(), out.data_ptr(),
                                        None if sum_out is None else sum_out.data_ptr(), x.shape[0],
                                        x.shape[1], self.config.rms_norm_eps, self.code, stream), "rms_norm")

    def forward_decode_batch(self, input_ids, block_tables, positions):
        """Logits of one decode step (native_qwen3.py:423-456)."""
        cfg, pool, w = self.config, self.pool, self.weights
        if input_ids.ndim != 1 or input_ids.dtype != torch.long or input_ids.numel() == 0:
            raise ValueError("input_ids must be a nonempty 1D int64 batch")
        if positions.ndim != 1 or positions.shape != input_ids.shape or positions.dtype != torch.long:
            raise ValueError("positions must be int64 with one value per request")
        if block_tables.ndim != 2 or block_tables.shape[0] != input_ids.shape[0]:
            raise ValueError("block_tables must be [batch, max_blocks]")
        if block_tables.dtype != torch.long or not block_tables.is_contiguous():
            raise ValueError("block_tables must be a contiguous int64 tensor")
        device = w.embed.device
        if input_ids.device != device or positions.device != device or block_tables.device != device:
            raise ValueError("decode inputs must be on the model device")
        capturing = torch.cuda.is_current_stream_capturing()
        if not capturing and (bool((positions < 0).any())
                              or bool((positions + 1 > cfg.max_position_embeddings).any())):
            raise ValueError("decode positions exceed model context")
        batch = input_ids.shape[0]
        hq, hkv, dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        shape = pool.shape
        stream = torch.cuda.current_stream(device).cuda_stream
        self._stage_begin(batch, block_tables, positions)
        if self.fused_projections and batch <= self.FUSED_MAX_BATCH:
            return self._forward_fused(input_ids, block_tables, positions, stream)
        x = F.embedding(input_ids, w.embed)
        cos, sin = self._rotary(positions)
        h = torch.empty_like(x)
        self._rms(x, None, w.layers[0].input_norm, h, None, stream)
        residual = x
        for index, layer in enumerate(w.layers):
            qkv = torch.mm(h, layer.qkv.t())
            q = torch.empty((batch, hq, dim), dtype=x.dtype, device=device)
            kc, vc, tables, pos, blocks, bs, width = self._append_target(index, block_tables, positions)
            _check(self.lib.minikv_qk_rope_append(
                qkv.data_ptr(), qkv.stride(0), layer.q_norm.data_ptr(), layer.k_norm.data_ptr(), cos.data_ptr(),
                sin.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), pos.data_ptr(),
                batch, hq, hkv, dim, blocks, bs, width, cfg.rms_norm_eps, self.code, stream), "qk_rope_append")
            attention = self._attend(index, q, block_tables, positions)
            o = torch.mm(attention.view(batch, hq * dim), layer.o.t())
            summed, normalized = torch.empty_like(x), torch.empty_like(x)
            self._rms(o, residual, layer.post_norm, normalized, summed, stream)
            gate_up = torch.mm(normalized, layer.gate_up.t())
            act = torch.empty((batch, cfg.intermediate_size), dtype=x.dtype, device=device)
            _check(self.lib.minikv_silu_mul(gate_up.data_ptr(), act.data_ptr(), batch, cfg.intermediate_size,
                                            self.code, stream), "silu_mul")
            down = torch.mm(act, layer.down.t())
            following = w.layers[index + 1].input_norm if index + 1 < len(w.layers) else w.norm
            residual, h = torch.empty_like(x), torch.empty_like(x)
            self._rms(down, summed, following, h, residual, stream)
        return torch.mm(h, w.lm_head.t())

    def _forward_fused(self, input_ids, block_tables, positions, stream):
        """The step on the fused tcgen05 projections (five launches per layer)."""
        cfg, pool, w, lib, code = self.config, self.pool, self.weights, self.lib, self.code
        batch, device = input_ids.shape[0], input_ids.device
        hq, hkv, dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        hidden, inter, eps = cfg.hidden_size, cfg.intermediate_size, cfg.rms_norm_eps
        shape = pool.shape
        x = F.embedding(input_ids, w.embed)
        cos, sin = self._rotary(positions)
        h = torch.empty_like(x)
        self._rms(x, None, w.layers[0].input_norm, h, None, stream)
        residual, sums = x, None  # sums: per-row partial sums of squares of `residual`
        for index, layer in enumerate(w.layers):
            qkv_w, o_w, gate_up_w, down_w = self._packed[index]
            q = torch.empty((batch, hq, dim), dtype=x.dtype, device=device)
            if sums is None:  # first layer: RMSNorm already applied
                source, ss_in, norm = h, None, None
            else:
                source, ss_in, norm = residual, sums.data_ptr(), layer.input_norm.data_ptr()
            kc, vc, tables, pos, blocks, bs, width = self._append_target(index, block_tables, positions)
            _check(lib.minikv_linear_qk_rope_append(
                source.data_ptr(), source.stride(0), ss_in, norm, eps, qkv_w.data_ptr(),
                layer.q_norm.data_ptr(), layer.k_norm.data_ptr(), cos.data_ptr(), sin.data_ptr(), q.data_ptr(),
                kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), pos.data_ptr(), batch, hidden, hq, hkv, dim,
                blocks, bs, width, code, stream), "linear_qk_rope_append")
            attention = self._attend(index, q, block_tables, positions)
            summed = torch.empty_like(x)
            summed_sums = torch.empty((hidden // 128, batch), dtype=torch.float32, device=device)
            _check(lib.minikv_linear_residual(
                attention.data_ptr(), hq * dim, o_w.data_ptr(), residual.data_ptr(), summed.data_ptr(),
                summed_sums.data_ptr(), batch, hq * dim, hidden, code, stream), "linear_residual(o)")
            act = torch.empty((batch, inter), dtype=x.dtype, device=device)
            _check(lib.minikv_linear_silu_mul(
                summed.data_ptr(), hidden, summed_sums.data_ptr(), layer.post_norm.data_ptr(), eps,
                gate_up_w.data_ptr(), act.data_ptr(), batch, hidden, inter, code, stream), "linear_silu_mul")
            residual = torch.empty_like(x)
            sums = torch.empty((hidden // 128, batch), dtype=torch.float32, device=device)
            _check(lib.minikv_linear_residual(
                act.data_ptr(), inter, down_w.data_ptr(), summed.data_ptr(), residual.data_ptr(),
                sums.data_ptr(), batch, inter, hidden, code, stream), "linear_residual(down)")
        h = torch.empty_like(x)
        self._rms(residual, None, w.norm, h, None, stream)
        return torch.mm(h, w.lm_head.t())

    # ------------------------------------------------------ KV pool access
    def _stage_begin(self, batch, block_tables, positions):
        """Per-step staging rows of the new tokens' K/V."""
        cfg = self.config
        device = positions.device
        shape = (batch, 1, cfg.num_key_value_heads, cfg.head_dim)
        self._stage_k = torch.empty(shape, dtype=self.weights.embed.dtype, device=device)
        self._stage_v = torch.empty_like(self._stage_k)
        key = (batch, device)
        if key not in self._stage_index:  # read-only index tensors: made once per batch size
            self._stage_index[key] = (torch.arange(batch, dtype=torch.long, device=device).view(batch, 1),
                                      torch.zeros(batch, dtype=torch.long, device=device))
        self._stage_tables, self._stage_pos = self._stage_index[key]

    def _append_target(self, index, block_tables, positions):
        """Where the q/k-norm + RoPE kernels write the new token's K/V: staging rows, one 1-token page
        per request (page b, offset 0).  The decode appends them to the pool."""
        return (self._stage_k, self._stage_v, self._stage_tables, self._stage_pos, self._stage_k.shape[0], 1, 1)

    def _attend(self, index, q, block_tables, positions):
        """Append (from the staging rows) and decode in one launch, chained: the tables, positions
        and the pool rows it reads predate the kernel just launched, which wrote only q and the
        staging rows, so the decode stages pool rows at once.  An fp8 pool quantises the new rows
        into their slots inside the same launch."""
        pool = self.pool
        batch = q.shape[0]
        rows = (batch, self.config.num_key_value_heads, self.config.head_dim)
        stage_k, stage_v = self._stage_k.view(rows), self._stage_v.view(rows)
        if not self.fp8:
            return paged_attention_with_append(q, pool.key[index], pool.value[index], block_tables, positions,
                                               stage_k, stage_v, pool.shape.block_size, validate=False,
                                               chained=True)
        return paged_attention_fp8_with_append(q, pool.key[index], pool.value[index], block_tables, positions,
                                               stage_k, stage_v, pool.shape.block_size, pool.k_scale, pool.v_scale,
                                               kv_format=pool.kv_format, validate=False, chained=True)

    def greedy(self, input_ids, block_tables, positions):
        """Greedy next token of every request (argmax of the step's logits)."""
        return greedy_ids(self.forward_decode_batch(input_ids, block_tables, positions))


class DecodeGraph:
    """A greedy decode step captured as one CUDA graph for a fixed batch and table width.

    The static inputs (``input_ids``, ``positions``, ``block_tables``) are
    refilled before every replay, as the reference's ``DecodeGraphBucket``
    does (``mini_engine/engine/cuda_graph.py:196-275``); the output is
    ``next_ids``.  The decode workspace of the capture stream is created by a
    warm-up step on that stream before capture.

    Two ways to fill the inputs:

    * :meth:`load` copies ready ``[batch]`` / ``[batch, table_width]`` tensors
      (host or device) into the static buffers;
    * with ``padding_pages`` (one private scratch page per batch row), the
      graph is a bucket that serves up to ``batch`` requests: :meth:`stage`
      packs one step's tokens, positions and per-request page lists into one
      pinned host buffer and makes one host-to-device copy, and the graph's
      first kernel (``minikv_build_decode_tables``) builds the fixed-shape
      inputs on the device -- the staging of cuda_graph.py:149-181 -- with the
      rows past the active requests decoding position 0 on their scratch page
      (cuda_graph.py:66-86).
    """

    def __init__(self, step: Qwen3DecodeStep, batch: int, table_width: int, *, warmup_tables=None,
                 padding_pages=None):
        device = step.weights.embed.device
        self.step = step
        self.device = device
        self.batch, self.table_width = batch, table_width
        self.input_ids = torch.zeros(batch, dtype=torch.long, device=device)
        self.positions = torch.zeros(batch, dtype=torch.long, device=device)
        self.block_tables = torch.full((batch, table_width), -1, dtype=torch.long, device=device)
        if warmup_tables is not None:
            self.block_tables.copy_(warmup_tables)
        self.staged = padding_pages is not None
        if self.staged:
            self._init_staging(padding_pages)
        self.stream = torch.cuda.Stream(device)
        self.graph = torch.cuda.CUDAGraph()
        self.stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(self.stream):
            # warm-up: allocates the stream's decode workspace and cuBLAS state outside the graph
            if self.staged:
                self._build_tables()
            step.greedy(self.input_ids, self.block_tables, self.positions)
        self.stream.synchronize()
        with torch.cuda.graph(self.graph, stream=self.stream):
            if self.staged:
                self._build_tables()
            self.next_ids = step.greedy(self.input_ids, self.block_tables, self.positions)
        torch.cuda.current_stream(device).wait_stream(self.stream)

    def _init_staging(self, padding_pages):
        pages = [int(p) for p in padding_pages][:self.batch]
        num_blocks = self.step.pool.shape.num_blocks
        if len(pages) < self.batch:
            raise ValueError("padding_pages must cover one private page per batch slot")
        if len(set(pages)) != self.batch or any(p < 0 or p >= num_blocks for p in pages):
            raise ValueError("padding slots require distinct scratch pages inside the cache")
        batch, width = self.batch, self.table_width
        self._padding = torch.tensor(pages, dtype=torch.long, device=self.device)
        # [active | tokens[batch] | positions[batch] | cu_blocks[batch + 1] | block ids ...]
        self._offsets = (0, 1, 1 + batch, 1 + 2 * batch, 2 + 3 * batch)
        size = 2 + 3 * batch + batch * width
        self._host = torch.zeros(size, dtype=torch.long, pin_memory=True)
        self._dev = torch.zeros(size, dtype=torch.long, device=self.device)
        self._host_np = self._host.numpy()
        self._copied = torch.cuda.Event()
        self._copy_pending = False

    def _build_tables(self):
        o, d = self._offsets, self._dev
        stream = _lib.stream_of(self.device)
        _check(self.step.lib.minikv_build_decode_tables(
            d[o[0]:].data_ptr(), d[o[1]:].data_ptr(), d[o[2]:].data_ptr(), d[o[3]:].data_ptr(), d[o[4]:].data_ptr(),
            self._padding.data_ptr(), self.batch, self.table_width, self.input_ids.data_ptr(),
            self.positions.data_ptr(), self.block_tables.data_ptr(), stream), "build_decode_tables")

    def load(self, input_ids, positions, block_tables):
        """Copy one step's metadata into the static buffers (host or device tensors)."""
        if self.staged:
            raise ValueError("a staged decode graph takes its inputs through stage()")
        self.input_ids.copy_(input_ids, non_blocking=True)
        self.positions.copy_(positions, non_blocking=True)
        self.block_tables.copy_(block_tables, non_blocking=True)

    def stage(self, tokens, positions, block_lists):
        """Stage one step of up to ``batch`` requests with one host-to-device copy.

        ``tokens`` and ``positions`` hold one int per request; ``block_lists``
        one sequence of physical page ids per request (1 .. table_width pages).
        """
        import numpy as np

        active = len(tokens)
        if active > self.batch or len(positions) != active or len(block_lists) != active:
            raise ValueError("staged requests exceed the graph's batch or have mismatched lengths")
        counts = [len(row) for row in block_lists]
        if any(n < 1 or n > self.table_width for n in counts):
            raise ValueError("each request needs 1 .. table_width pages")
        if self._copy_pending:  # the previous copy may still read the pinned buffer
            self._copied.synchronize()
        o, h = self._offsets, self._host_np
        h[0] = active
        h[o[1]:o[1] + active] = tokens
        h[o[2]:o[2] + active] = positions
        cu = np.zeros(active + 1, dtype=np.int64)
        np.cumsum(counts, out=cu[1:])
        h[o[3]:o[3] + active + 1] = cu
        total = int(cu[-1])
        if total:
            h[o[4]:o[4] + total] = np.concatenate([np.asarray(row, dtype=np.int64) for row in block_lists])
        used = o[4] + total
        self._dev[:used].copy_(self._host[:used], non_blocking=True)
        self._copied.record(torch.cuda.current_stream(self.device))
        self._copy_pending = True

    def replay(self):
        self.graph.replay()
        return self.next_ids
