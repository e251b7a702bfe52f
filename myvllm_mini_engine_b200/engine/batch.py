"""Ragged prefill batch metadata built on the device.

``PrefillBatch.from_sequences`` keeps the signature, validation rules, error
messages and outputs of ``mini_engine/engine/batch.py:67-137``, but the
per-token work moves to the GPU: the host validates at *page* granularity
(numpy over requests and pages, never a Python loop over tokens), packs the
per-request inputs into one pinned buffer, issues one host-to-device copy and
one ``minikv_build_prefill_metadata`` launch that expands positions, slot
mapping, offsets, context lengths and the -1 padded block tables.  All seven
outputs are views of one device allocation.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from numbers import Integral

import numpy as np
import torch

from .. import _lib

_INT64_MIN, _INT64_MAX = -(1 << 63), (1 << 63) - 1


def _integers(values, name):
    """batch.py:9-22, with a numpy fast path for integer arrays."""
    if isinstance(values, torch.Tensor):
        if values.ndim != 1 or values.dtype != torch.int64:
            raise ValueError(f"{name} must be a 1D int64 tensor")
        return values.detach().cpu().numpy().astype(np.int64, copy=False)
    if isinstance(values, np.ndarray) and values.ndim == 1 and values.dtype.kind in "iu":
        return values.astype(np.int64)
    try:
        result = tuple(values)
    except TypeError as error:
        raise ValueError(f"{name} must be a sequence of integers") from error
    if any(isinstance(value, bool) or not isinstance(value, Integral) for value in result):
        raise ValueError(f"{name} must contain integers")
    if any(value < _INT64_MIN or value > _INT64_MAX for value in result):
        raise ValueError(f"{name} values must fit int64")
    return np.asarray(result, dtype=np.int64).reshape(-1)


def _signature(tensor):
    return (tensor.data_ptr(), tensor._version, tuple(tensor.shape), tuple(tensor.stride()),
            tensor.dtype, tensor.device)


@dataclass(frozen=True)
class PrefillBatch:
    """Read-only metadata for nonempty query chunks (batch.py:31-57)."""

    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    cu_seqlens_q: torch.Tensor
    query_starts: torch.Tensor
    context_lens: torch.Tensor
    block_tables: torch.Tensor
    query_lengths: tuple[int, ...]
    query_offsets: tuple[int, ...]
    starts: tuple[int, ...]
    block_ids: tuple[tuple[int, ...], ...]
    block_size: int
    num_blocks: int
    _token_values: np.ndarray = field(repr=False, compare=False)
    _tensor_signatures: tuple = field(repr=False, compare=False)

    _TENSOR_NAMES = ("input_ids", "positions", "slot_mapping", "cu_seqlens_q",
                     "query_starts", "context_lens", "block_tables")

    @property
    def batch_size(self):
        return len(self.query_lengths)

    @property
    def num_tokens(self):
        return self.query_offsets[-1]

    @classmethod
    def from_sequences(cls, token_sequences, block_tables, query_starts, *, block_size, num_blocks, device):
        for name, value in (("block_size", block_size), ("num_blocks", num_blocks)):
            if isinstance(value, bool) or not isinstance(value, Integral) or value <= 0:
                raise ValueError(f"{name} must be a positive integer")
        block_size, num_blocks = int(block_size), int(num_blocks)
        try:
            sequences = [_integers(values, "token sequence") for values in token_sequences]
        except TypeError as error:
            raise ValueError("token_sequences must contain query sequences") from error
        if not sequences or any(values.size == 0 for values in sequences):
            raise ValueError("prefill batch requires nonempty query sequences")
        starts = _integers(query_starts, "query_starts")
        if isinstance(block_tables, torch.Tensor):
            if block_tables.ndim != 2 or block_tables.dtype != torch.int64:
                raise ValueError("block_tables must be a 2D int64 tensor")
            block_tables = list(block_tables.detach().cpu().numpy())
        tables = [_integers(values, "block table") for values in block_tables]
        if len(starts) != len(sequences) or len(tables) != len(sequences):
            raise ValueError("queries, query_starts and block_tables must have equal batch size")

        clean, lengths = [], []
        readers: dict[int, set] = {}
        written: dict[int, list] = {}   # page -> [(request, first_slot, end_slot)]
        for request, (tokens, table, start) in enumerate(zip(sequences, tables, starts.tolist())):
            if start < 0:                                   # batch.py:89-107, same order
                raise ValueError("query_starts must be nonnegative")
            if (tokens < 0).any():
                raise ValueError("token IDs must be nonnegative")
            pad = np.flatnonzero(table == -1)
            first_padding = int(pad[0]) if pad.size else table.size
            if (table[first_padding:] != -1).any():
                raise ValueError("block table padding -1 must be trailing")
            table = table[:first_padding]
            if ((table < 0) | (table >= num_blocks)).any():
                raise ValueError("physical block ID out of range")
            if np.unique(table).size != table.size:
                raise ValueError("a request block table cannot contain duplicate physical pages")
            end = start + int(tokens.size)
            if end > table.size * block_size:
                raise ValueError("query range exceeds supplied block table capacity")
            for page in table.tolist():
                readers.setdefault(page, set()).add(request)
            # Writes of this request, page by page (batch.py:110-118 per token).
            for index in range(start // block_size, (end - 1) // block_size + 1):
                page = int(table[index])
                lo = max(start, index * block_size) - index * block_size
                hi = min(end, (index + 1) * block_size) - index * block_size
                for _, a, b in written.get(page, ()):
                    if lo < b and a < hi:
                        raise ValueError("prefill batch contains duplicate writable KV slots")
                written.setdefault(page, []).append((request, lo, hi))
            lengths.append(int(tokens.size))
            clean.append(table)
        for page, writes in written.items():                 # batch.py:124-126
            if len(readers[page] | {request for request, _, _ in writes}) > 1:
                raise ValueError("prefill cannot write a physical page shared by requests")

        batch = len(sequences)
        width = max(table.size for table in clean)
        offsets = np.zeros(batch + 1, dtype=np.int64)
        np.cumsum(lengths, out=offsets[1:])
        cu_blocks = np.zeros(batch + 1, dtype=np.int64)
        np.cumsum([table.size for table in clean], out=cu_blocks[1:])
        total = int(offsets[-1])
        token_values = np.concatenate(sequences)
        staging = np.concatenate([starts, offsets, cu_blocks, np.concatenate(clean), token_values])
        device = torch.device(device)
        with torch.inference_mode(False):
            sizes = (total, total, total, batch + 1, batch, batch, batch * width)
            out = torch.empty(sum(sizes), dtype=torch.int64, device=device)
            views = list(torch.split(out, sizes))
            views[-1] = views[-1].view(batch, width)
            if device.type == "cuda":
                host = torch.from_numpy(staging).pin_memory()
                staged = torch.empty_like(host, device=device)
                staged.copy_(host, non_blocking=True)
                o_starts, o_cu_q = 0, batch
                o_cu_b = o_cu_q + batch + 1
                o_blocks = o_cu_b + batch + 1
                o_tokens = o_blocks + int(cu_blocks[-1])
                base = staged.data_ptr()
                lib = _lib.load()
                with torch.cuda.device(device):
                    status = lib.minikv_build_prefill_metadata(
                        base + 8 * o_starts, base + 8 * o_cu_q, base + 8 * o_cu_b, base + 8 * o_blocks,
                        base + 8 * o_tokens, batch, total, width, block_size,
                        *(v.data_ptr() for v in views), _lib.stream_of(device))
                _lib.check(status, "PrefillBatch.from_sequences")
                # No sync: torch's pinned-memory allocator keeps `host` until the
                # copy completes, and `staged` is reused only by later work on
                # this stream.
            else:
                raise ValueError("device-side prefill metadata needs a CUDA device")
        return cls(*views, tuple(lengths), tuple(int(x) for x in offsets), tuple(int(s) for s in starts),
                   tuple(tuple(int(p) for p in table) for table in clean), block_size, num_blocks,
                   token_values, tuple(map(_signature, views)))

    def validate(self, *, block_size, num_blocks, device, max_position_embeddings, vocab_size):
        """Validate the public execution boundary (batch.py:139-155)."""
        if self.block_size != block_size or self.num_blocks != num_blocks:
            raise ValueError("prefill metadata does not match KV cache geometry")
        device = torch.device(device)
        tensors = tuple(getattr(self, name) for name in self._TENSOR_NAMES)
        if len(self._tensor_signatures) != len(tensors):
            raise ValueError("construct prefill metadata with PrefillBatch.from_sequences")
        if any(not isinstance(tensor, torch.Tensor) or tensor.dtype != torch.int64
               or tensor.device != device or not tensor.is_contiguous() for tensor in tensors):
            raise ValueError("prefill metadata must be contiguous int64 tensors on the cache device")
        if tuple(map(_signature, tensors)) != self._tensor_signatures:
            raise ValueError("prefill metadata was modified; rebuild it with from_sequences")
        if any(start + length > max_position_embeddings for start, length in zip(self.starts, self.query_lengths)):
            raise ValueError("prefill query range exceeds model context limit")
        if self._token_values.size and int(self._token_values.max()) >= vocab_size:
            raise ValueError("prefill token ID exceeds model vocabulary")
