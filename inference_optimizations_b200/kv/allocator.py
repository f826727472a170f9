"""Page allocation for the paged KV pools.

`PageAllocator` hands out fixed-size physical pages (64 tokens) from a LIFO free list; page 0 of every pool is
reserved as the dummy page that padded (CUDA-graph filler) requests point at, so a padded row never touches live
data.  `PageTable` is the device-side [max_requests, max_pages] int32 map from logical page to physical page with a
pinned host mirror: the scheduler edits the host copy and `sync()` issues one H2D copy per step (graph-safe: the device
tensor's address never changes).  Reference behaviour: SGLang's token-to-KV pool allocator with page size 64
(`kv-cache-4bit/glm-kv4/glm_kv4_engine.py:90-141`); the sliding-window release is this framework's own.
"""
from __future__ import annotations

from typing import Optional

import torch

DUMMY_PAGE = 0


class OutOfPages(RuntimeError):
    pass


class PageAllocator:
    def __init__(self, num_pages: int, reserved: int = 1):
        if num_pages <= reserved:
            raise ValueError("pool too small")
        self.num_pages = num_pages
        self.reserved = reserved
        self._free = list(range(num_pages - 1, reserved - 1, -1))

    @property
    def free(self) -> int:
        return len(self._free)

    @property
    def used(self) -> int:
        return self.num_pages - self.reserved - len(self._free)

    def alloc(self, n: int) -> list[int]:
        if n > len(self._free):
            raise OutOfPages(f"need {n} pages, {len(self._free)} free")
        out = self._free[-n:] if n else []
        del self._free[len(self._free) - n:]
        return out[::-1]

    def release(self, pages: list[int]) -> None:
        for p in pages:
            if p >= self.reserved:
                self._free.append(p)

    def reset(self) -> None:
        """Every page free again, in the initial order (only with no request holding pages): a re-registered set of
        requests then gets the same physical pages as the first time."""
        self._free = list(range(self.num_pages - 1, self.reserved - 1, -1))


class PageTable:
    """Device page table with a pinned host mirror."""

    def __init__(self, max_requests: int, max_pages: int, device):
        self.max_requests = max_requests
        self.max_pages = max_pages
        pin = torch.cuda.is_available() and str(device).startswith("cuda")
        self.host = torch.full((max_requests, max_pages), DUMMY_PAGE, dtype=torch.int32, pin_memory=pin)
        self.dev = self.host.to(device) if str(device) != "cpu" else self.host.clone()
        self._dirty: set[int] = set()
        self.bytes_synced = 0

    def set(self, req: int, logical: int, phys: int) -> None:
        self.host[req, logical] = phys
        self._dirty.add(req)

    def clear(self, req: int) -> None:
        self.host[req].fill_(DUMMY_PAGE)
        self._dirty.add(req)

    def sync(self) -> None:
        """Copy dirty rows to the device (one copy of the covering row range)."""
        if not self._dirty:
            return
        lo, hi = min(self._dirty), max(self._dirty) + 1
        self.dev[lo:hi].copy_(self.host[lo:hi], non_blocking=True)
        self._dirty.clear()
        self.bytes_synced += (hi - lo) * self.max_pages * 4


class RequestPages:
    """Pages of one request in one pool kind.  With `window` > 0, pages wholly before the attention window of the
    next query are released as the sequence advances (sliding-window layers keep O(window) memory)."""

    def __init__(self, alloc: PageAllocator, table: PageTable, slot: int, page: int = 64, window: int = 0,
                 slack: int = 0):
        self.alloc, self.table, self.slot, self.page = alloc, table, slot, page
        self.window, self.slack = window, slack
        self.pages: dict[int, int] = {}
        self.length = 0
        self.high = 0          # logical pages [0, high) have been allocated at some point

    def ensure(self, new_len: int) -> None:
        """Make positions [0, new_len) addressable (allocating pages after the high-water mark)."""
        need = (new_len + self.page - 1) // self.page
        todo = list(range(self.high, need))
        if todo:
            got = self.alloc.alloc(len(todo))
            for lp, pp in zip(todo, got):
                self.pages[lp] = pp
                self.table.set(self.slot, lp, pp)
            self.high = need
        self.length = max(self.length, new_len)

    def trim(self, next_query_pos: int) -> None:
        """Release pages no query at or after `next_query_pos` can see (sliding window only)."""
        if self.window <= 0:
            return
        first_visible = next_query_pos - self.window + 1 - self.slack
        dead = [lp for lp in self.pages if (lp + 1) * self.page <= first_visible]
        if dead:
            self.alloc.release([self.pages.pop(lp) for lp in dead])
            for lp in dead:
                self.table.set(self.slot, lp, DUMMY_PAGE)

    def slot_of(self, pos: int) -> int:
        return self.pages[pos // self.page] * self.page + pos % self.page

    def free(self) -> None:
        self.alloc.release(list(self.pages.values()))
        self.pages.clear()
        self.table.clear(self.slot)
        self.length = 0
        self.high = 0

    def truncate(self, new_len: int) -> None:
        """Shrink the logical length (rejected speculative tokens); pages stay allocated."""
        self.length = min(self.length, new_len)


def pages_for(tokens: int, page: int = 64) -> int:
    return (tokens + page - 1) // page


def max_pages_needed(max_seq: int, page: int = 64, extra: Optional[int] = None) -> int:
    return pages_for(max_seq + (extra or 0), page)
