"""KV-cache page allocator.

Pages are fixed-size token blocks of the engine's KV pool.  Page 0 is reserved
as a trash page: idle decode rows in a captured CUDA graph write their K/V
there, so they can never touch a live request's pages.  The allocator is a
LIFO free list (recently freed pages are reused first, which keeps the
working set warm in L2); the native version (``meshy_b200._native``
``PageAllocator``) implements the same interface in C++ for the
scheduler-side hot loop.
"""

from __future__ import annotations


class BlockManager:
    def __init__(self, n_pages: int, page_size: int):
        if n_pages < 2:
            raise ValueError("need at least 2 KV pages (page 0 is reserved)")
        self.n_pages = n_pages
        self.page_size = page_size
        self._free = list(range(n_pages - 1, 0, -1))

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> list[int] | None:
        if n <= 0:
            return []
        if n > len(self._free):
            return None
        out = self._free[-n:][::-1]
        del self._free[-n:]
        return out

    def free(self, pages) -> None:
        self._free.extend(reversed(list(pages)))


__all__ = ["BlockManager"]
