"""CPU oracle: ragged-batch and decode-graph metadata.  Test infrastructure only.

Restates
  * ``mini_engine/engine/batch.py:67-137`` -- ``PrefillBatch.from_sequences``:
    validation (messages kept verbatim) and the per-token construction of
    ``input_ids``, ``positions`` (``start + i``), ``slot_mapping``
    (``table[p // bs] * bs + p % bs``), ``cu_seqlens_q``, ``query_starts``,
    ``context_lens`` (``start + len``) and ``block_tables`` (-1 padded to the
    widest request);
  * ``mini_engine/engine/cuda_graph.py:149-181`` (``_stage_metadata``) with the
    padding rows of :66-86 and :187-194 -- the fixed-shape decode metadata of a
    CUDA-graph bucket: inactive rows get token 0, position 0 and a private
    scratch page in column 0, every missing column is -1.
Pure Python integers; results are plain lists.
"""

from __future__ import annotations

from numbers import Integral


def _integers(values, name):
    # batch.py:9-22 (tensor inputs are converted by the caller)
    try:
        result = tuple(values)
    except TypeError as error:
        raise ValueError(f"{name} must be a sequence of integers") from error
    if any(isinstance(value, bool) or not isinstance(value, Integral) for value in result):
        raise ValueError(f"{name} must contain integers")
    if any(value < -(1 << 63) or value >= (1 << 63) for value in result):
        raise ValueError(f"{name} values must fit int64")
    return tuple(int(value) for value in result)


def prefill_metadata(token_sequences, block_tables, query_starts, *, block_size, num_blocks):
    """Return the seven metadata lists of ``PrefillBatch.from_sequences`` (batch.py:67-137)."""
    for name, value in (("block_size", block_size), ("num_blocks", num_blocks)):
        if isinstance(value, bool) or not isinstance(value, Integral) or value <= 0:
            raise ValueError(f"{name} must be a positive integer")
    sequences = tuple(_integers(values, "token sequence") for values in token_sequences)
    if not sequences or any(not values for values in sequences):
        raise ValueError("prefill batch requires nonempty query sequences")
    starts = _integers(query_starts, "query_starts")
    tables = tuple(_integers(values, "block table") for values in block_tables)
    if len(starts) != len(sequences) or len(tables) != len(sequences):
        raise ValueError("queries, query_starts and block_tables must have equal batch size")
    offsets, token_ids, positions, slots, contexts, clean = [0], [], [], [], [], []
    readers, writers, written = {}, {}, set()
    for request, (tokens, table, start) in enumerate(zip(sequences, tables, starts)):  # :88-123
        if start < 0:
            raise ValueError("query_starts must be nonnegative")
        if any(token < 0 for token in tokens):
            raise ValueError("token IDs must be nonnegative")
        first_padding = next((i for i, page in enumerate(table) if page == -1), len(table))
        if any(page != -1 for page in table[first_padding:]):
            raise ValueError("block table padding -1 must be trailing")
        table = table[:first_padding]
        if any(page < 0 or page >= num_blocks for page in table):
            raise ValueError("physical block ID out of range")
        if len(set(table)) != len(table):
            raise ValueError("a request block table cannot contain duplicate physical pages")
        end = start + len(tokens)
        if end > len(table) * block_size:
            raise ValueError("query range exceeds supplied block table capacity")
        for page in table:
            readers.setdefault(page, set()).add(request)
        for position in range(start, end):
            page = table[position // block_size]
            slot = page * block_size + position % block_size
            if slot in written:
                raise ValueError("prefill batch contains duplicate writable KV slots")
            written.add(slot)
            writers.setdefault(page, set()).add(request)
            positions.append(position)
            slots.append(slot)
        offsets.append(offsets[-1] + len(tokens))
        token_ids.extend(tokens)
        contexts.append(end)
        clean.append(table)
    for page, who in writers.items():  # :124-126
        if len(readers[page] | who) > 1:
            raise ValueError("prefill cannot write a physical page shared by requests")
    width = max(map(len, clean))
    padded = [list(table) + [-1] * (width - len(table)) for table in clean]  # :129
    return {"input_ids": token_ids, "positions": positions, "slot_mapping": slots,
            "cu_seqlens_q": offsets, "query_starts": list(starts), "context_lens": contexts,
            "block_tables": padded}


def decode_bucket_metadata(tokens, positions, block_tables, *, batch_size, max_blocks, padding_pages):
    """Staged decode metadata of a graph bucket (cuda_graph.py:149-181, :66-86, :187-194).

    Returns ``input_ids [batch_size]``, ``positions [batch_size]`` and
    ``block_tables [batch_size][max_blocks]``: active rows first, then padding
    rows that decode position 0 on their private scratch page.
    """
    active = len(tokens)
    ids = [0] * batch_size
    pos = [0] * batch_size
    ids[:active] = list(tokens)
    pos[:active] = list(positions)
    tables = [[-1] * max_blocks for _ in range(batch_size)]
    for row in range(batch_size):
        tables[row][0] = padding_pages[row]
    for row, table in enumerate(block_tables):  # rows hold 1..max_blocks pages (:106-108)
        tables[row][:len(table)] = list(table)
    return {"input_ids": ids, "positions": pos, "block_tables": tables}
