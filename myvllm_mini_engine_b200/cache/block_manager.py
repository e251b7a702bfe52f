"""Host-side KV page allocator with copy-on-write.

Same API and behaviour as ``mini_engine/cache/block_manager.py`` (LIFO free
list, per-page refcounts, prefix attach/pin, grow/truncate/release; :10-166),
which stays on the host.  New here: :meth:`BlockManager.copy_on_write` and
:meth:`BlockManager.prepare_write`, the host half of copy-on-write -- before a
request writes into a page whose refcount is above one, it gets a private
copy: a fresh page is allocated, the request's table entry is patched, the
shared page loses one reference, and the ``(src, dst)`` pair is returned for
the device copy (``kernels.data.copy_blocks``).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class BlockTable:
    request_id: str
    block_ids: tuple[int, ...]


class BlockManager:
    """Fixed-size KV block allocator (block_manager.py:10-166) plus copy-on-write."""

    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free: list[int] = list(range(num_blocks - 1, -1, -1))
        self._owned: dict[str, list[int]] = {}
        self._refcounts: list[int] = [0] * num_blocks

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    @property
    def used_blocks(self) -> int:
        return self.num_blocks - self.free_blocks

    def blocks_required(self, token_count: int) -> int:
        if token_count < 0:
            raise ValueError("token_count cannot be negative")
        return (token_count + self.block_size - 1) // self.block_size

    def can_allocate(self, token_count: int) -> bool:
        return self.blocks_required(token_count) <= self.free_blocks

    def _take(self, count: int) -> list[int]:
        blocks = [self._free.pop() for _ in range(count)]
        for block in blocks:
            self._refcounts[block] = 1
        return blocks

    def allocate(self, request_id: str, token_count: int) -> list[int]:
        if request_id in self._owned:
            raise ValueError(f"request already owns blocks: {request_id}")
        count = self.blocks_required(token_count)
        if count > self.free_blocks:
            raise MemoryError(f"need {count} blocks, only {self.free_blocks} free")
        self._owned[request_id] = self._take(count)
        return list(self._owned[request_id])

    def _check_attachable(self, blocks):
        for block in blocks:
            if block < 0 or block >= self.num_blocks or self._refcounts[block] <= 0:
                raise ValueError(f"cannot attach unallocated block: {block}")

    def allocate_with_prefix(self, request_id: str, token_count: int, prefix_block_ids) -> list[int]:
        """Attach cached prefix pages and allocate only the suffix pages (:55-82)."""
        if request_id in self._owned:
            raise ValueError(f"request already owns blocks: {request_id}")
        prefix = list(prefix_block_ids)
        if len(set(prefix)) != len(prefix):
            raise ValueError("prefix pages must be distinct")
        required = self.blocks_required(token_count)
        if len(prefix) > required:
            raise ValueError("prefix has more blocks than the request needs")
        self._check_attachable(prefix)
        suffix_count = required - len(prefix)
        if suffix_count > self.free_blocks:
            raise MemoryError(f"need {suffix_count} blocks, only {self.free_blocks} free")
        for block in prefix:
            self._refcounts[block] += 1
        self._owned[request_id] = prefix + self._take(suffix_count)
        return list(self._owned[request_id])

    def attach(self, request_id: str, block_ids) -> list[int]:
        if request_id in self._owned:
            raise ValueError(f"request already owns blocks: {request_id}")
        blocks = list(block_ids)
        if len(set(blocks)) != len(blocks):
            raise ValueError("attached pages must be distinct")
        self._check_attachable(blocks)
        for block in blocks:
            self._refcounts[block] += 1
        self._owned[request_id] = blocks
        return list(blocks)

    def pin(self, block_ids) -> None:
        for block in block_ids:
            if block < 0 or block >= self.num_blocks or self._refcounts[block] <= 0:
                raise ValueError(f"cannot pin unallocated block: {block}")
        for block in block_ids:
            self._refcounts[block] += 1

    def unpin(self, block_ids) -> None:
        for block in block_ids:
            self._decrement(block)

    def _decrement(self, block: int) -> None:
        if block < 0 or block >= self.num_blocks or self._refcounts[block] <= 0:
            raise ValueError(f"block is not retained: {block}")
        self._refcounts[block] -= 1
        if self._refcounts[block] == 0:
            self._free.append(block)

    def grow(self, request_id: str, token_count: int) -> list[int]:
        if request_id not in self._owned:
            return self.allocate(request_id, token_count)
        current = self._owned[request_id]
        needed = self.blocks_required(token_count) - len(current)
        if needed <= 0:
            return list(current)
        if needed > self.free_blocks:
            raise MemoryError(f"need {needed} additional blocks, only {self.free_blocks} free")
        current.extend(self._take(needed))
        return list(current)

    def release(self, request_id: str) -> None:
        blocks = self._owned.pop(request_id, None)
        if blocks is None:
            return
        for block in blocks:
            self._decrement(block)

    def truncate(self, request_id: str, keep_tokens: int) -> list[int]:
        count = self.blocks_required(keep_tokens)
        if request_id not in self._owned:
            raise KeyError(request_id)
        current = self._owned[request_id]
        if count > len(current):
            raise ValueError("truncate cannot grow a block table")
        removed = current[count:]
        del current[count:]
        for block in removed:
            self._decrement(block)
        return list(current)

    def refcount(self, block_id: int) -> int:
        if block_id < 0 or block_id >= self.num_blocks:
            raise IndexError(block_id)
        return self._refcounts[block_id]

    def table(self, request_id: str) -> BlockTable:
        if request_id not in self._owned:
            raise KeyError(request_id)
        return BlockTable(request_id, tuple(self._owned[request_id]))

    # ----------------------------------------------------------- copy-on-write
    def copy_on_write(self, request_id: str, block_index: int) -> tuple[int, int] | None:
        """Give ``request_id`` a private copy of its page ``block_index`` if it is shared.

        Returns ``(src, dst)`` for the device copy, or None when the page is
        already private (refcount 1).  The shared page keeps its other
        references (other requests, prefix-cache pins).
        """
        if request_id not in self._owned:
            raise KeyError(request_id)
        table = self._owned[request_id]
        if not 0 <= block_index < len(table):
            raise IndexError(block_index)
        src = table[block_index]
        if self._refcounts[src] <= 1:
            return None
        if not self._free:
            raise MemoryError("need 1 block for copy-on-write, none free")
        dst = self._take(1)[0]
        table[block_index] = dst
        self._decrement(src)
        return src, dst

    def prepare_write(self, request_id: str, start: int, end: int) -> list[tuple[int, int]]:
        """Copy-on-write every shared page that positions ``[start, end)`` of the request touch."""
        if start < 0 or end < start:
            raise ValueError("invalid write range")
        if end == start:
            return []
        first, last = start // self.block_size, (end - 1) // self.block_size
        pairs = []
        for index in range(first, last + 1):
            pair = self.copy_on_write(request_id, index)
            if pair is not None:
                pairs.append(pair)
        return pairs
