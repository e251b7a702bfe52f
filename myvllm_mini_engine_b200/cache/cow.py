"""Copy-on-write of shared KV pages, acting on the reference engine's own allocator.

The page allocator stays the reference's ``BlockManager``
(``mini_engine/cache/block_manager.py:10-166``): a LIFO free list ``_free``,
per-page reference counts ``_refcounts`` and each request's page list in
``_owned[request_id]``.  The reference shares prefix pages by reference count
(``allocate_with_prefix``/``attach``/``pin``) but never copies one, so a request
whose next chunk starts inside a shared page cannot write it
(``PrefillBatch.from_sequences`` rejects the batch, batch.py:126-128).

The two functions below add the missing fork.  They take any allocator with
those three attributes and ``block_size``; ``integration.install`` also binds
them as ``BlockManager.copy_on_write`` / ``BlockManager.prepare_write``.  The
device half is :func:`myvllm_mini_engine_b200.kernels.data.copy_blocks`, which
copies each returned ``(src, dst)`` page across every layer of the K and V pools.
"""

from __future__ import annotations


def copy_on_write(manager, request_id: str, block_index: int) -> tuple[int, int] | None:
    """Give ``request_id`` a private copy of entry ``block_index`` of its page list, if that page is shared.

    A page is shared when its reference count is above one (other requests or
    a prefix-cache pin hold it).  Then one page is taken from the free list
    (reference count 1) and put in the request's list in place of the shared
    one, which loses this request's reference.  Returns ``(src, dst)`` for the
    device copy, or None when the page was already private.  Raises KeyError
    for an unknown request, IndexError for an entry outside its list and
    MemoryError when no page is free (the allocator is then unchanged).
    """
    pages = manager._owned.get(request_id)
    if pages is None:
        raise KeyError(request_id)
    if not 0 <= block_index < len(pages):
        raise IndexError(block_index)
    shared = pages[block_index]
    counts = manager._refcounts
    if counts[shared] <= 1:
        return None
    if not manager._free:
        raise MemoryError("need 1 block for copy-on-write, none free")
    fresh = manager._free.pop()
    counts[fresh] = 1
    pages[block_index] = fresh
    counts[shared] -= 1  # stays >= 1: the other holders keep it, so it never returns to the free list here
    return shared, fresh


def prepare_write(manager, request_id: str, start: int, end: int) -> list[tuple[int, int]]:
    """Fork every shared page that logical positions ``[start, end)`` of ``request_id`` fall in.

    Call before scattering a chunk's K/V; apply the returned pairs with
    ``copy_blocks`` on the device before the scatter, and rebuild the request's
    block table from the allocator.
    """
    if start < 0 or end < start:
        raise ValueError("invalid write range")
    if end == start:
        return []
    size = manager.block_size
    forks = (copy_on_write(manager, request_id, index) for index in range(start // size, (end - 1) // size + 1))
    return [pair for pair in forks if pair is not None]
