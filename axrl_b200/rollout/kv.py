"""Block-manager factory for the paged KV cache.

The native implementation lives in ``csrc/runtime/block_manager.cpp`` (module
``axrl_b200._runtime``).  When the module has not been built yet (fresh
checkout on a CPU-only machine) it is built on first use with g++; the pure
Python :class:`PyBlockManager` (same semantics, used to cross-check the native
one in tests) is the last resort.
"""

from __future__ import annotations

from collections import OrderedDict

from axrl_b200.ops import _ext


def runtime_module():  # noqa: ANN201
    try:
        return _ext.load("_runtime")
    except Exception:  # noqa: BLE001
        from axrl_b200.csrc.build import build

        build(only="_runtime")
        return _ext.load("_runtime")


def make_block_manager(num_pages: int, page_size: int, prefer_native: bool = True):  # noqa: ANN201
    if prefer_native:
        try:
            return runtime_module().BlockManager(num_pages, page_size)
        except Exception:  # noqa: BLE001
            pass
    return PyBlockManager(num_pages, page_size)


def _mix64(h: int, v: int) -> int:
    M = (1 << 64) - 1
    z = (h ^ ((v + 0x9E3779B97F4A7C15 + ((h << 6) & M) + (h >> 2)) & M)) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


class PyBlockManager:
    """Pure-Python twin of the native BlockManager (identical hashing and eviction order)."""

    def __init__(self, num_pages: int, page_size: int) -> None:
        self.page_size, self.num_pages = page_size, num_pages
        self.ref = [0] * num_pages
        self.free = list(range(num_pages - 1, -1, -1))
        self.lru: OrderedDict[int, None] = OrderedDict()
        self.index: dict[int, int] = {}
        self.hash_of = [0] * num_pages
        self.cached = [False] * num_pages

    def num_available(self) -> int:
        return len(self.free) + len(self.lru)

    def num_free(self) -> int:
        return len(self.free)

    def num_cached(self) -> int:
        return len(self.index)

    def allocate(self, n: int) -> list[int]:
        if n > self.num_available():
            raise RuntimeError("KV cache out of pages")
        out = []
        for _ in range(n):
            if not self.free:
                p, _ = self.lru.popitem(last=False)
                del self.index[self.hash_of[p]]
                self.cached[p] = False
                self.free.append(p)
            p = self.free.pop()
            self.ref[p] = 1
            out.append(p)
        return out

    def incref(self, pages: list[int]) -> None:
        for p in pages:
            if self.ref[p] == 0 and self.cached[p]:
                del self.lru[p]
            self.ref[p] += 1

    def release(self, pages: list[int]) -> None:
        for p in pages:
            if self.ref[p] <= 0:
                raise RuntimeError("double free of KV page")
            self.ref[p] -= 1
            if self.ref[p] == 0:
                if self.cached[p]:
                    self.lru[p] = None
                else:
                    self.free.append(p)

    def _page_hash(self, h: int, t: list[int], i: int) -> int:
        for j in range(i * self.page_size, (i + 1) * self.page_size):
            h = _mix64(h, t[j] & ((1 << 64) - 1))
        return _mix64(h, 0xC0FFEE + i)

    def match_prefix(self, tokens: list[int]) -> tuple[list[int], int]:
        pages, h = [], 0
        for i in range(len(tokens) // self.page_size):
            h = self._page_hash(h, tokens, i)
            if h not in self.index:
                break
            pages.append(self.index[h])
        self.incref(pages)
        return pages, len(pages) * self.page_size

    def insert(self, tokens: list[int], pages: list[int]) -> None:
        h = 0
        for i in range(min(len(tokens) // self.page_size, len(pages))):
            h = self._page_hash(h, tokens, i)
            p = pages[i]
            if h in self.index or self.cached[p]:
                continue
            self.index[h] = p
            self.hash_of[p] = h
            self.cached[p] = True

    def clear_cache(self) -> None:
        for p in list(self.lru):
            self.cached[p] = False
            self.free.append(p)
        self.lru.clear()
        for p in self.index.values():
            self.cached[p] = False
        self.index.clear()

    def stats(self) -> dict:
        return {"num_pages": self.num_pages, "free": len(self.free), "cached": len(self.index), "evictable": len(self.lru)}
