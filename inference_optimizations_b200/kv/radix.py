"""Radix prefix cache over KV pages: a tree whose edges are whole 64-token pages of token ids, each node owning the
physical page that holds those tokens' KV.  New requests reuse the longest cached prefix of their prompt (read-only:
a request only writes positions after its reused prefix, which always start on a fresh page); finished requests
donate their full pages; unreferenced leaves are evicted least-recently-used when the allocator runs short.
SGLang's radix cache is what the reference serves with (its DCP / PD patches keep it working, e.g. the decode-side
radix cache of `parallelism/README.md:17-27`); this is a page-granular tree of its own."""
from __future__ import annotations

import itertools
from typing import Optional


class _Node:
    __slots__ = ("children", "page", "ref", "last", "parent", "key", "state")

    def __init__(self, parent: Optional["_Node"], key: Optional[tuple], page: int):
        self.children: dict = {}
        self.page, self.ref, self.parent, self.key = page, 0, parent, key
        self.last = 0
        self.state = None                   # hybrid models: recurrent state after this node's last token


class RadixCache:
    def __init__(self, alloc, page: int = 64):
        self.alloc, self.page = alloc, page
        self.root = _Node(None, None, -1)
        self.clock = itertools.count(1)
        self.held = 0                       # pages owned by the tree
        self.hits = self.lookups = 0
        self.stateful: set = set()          # nodes holding a recurrent state (hybrid models)

    def _chunks(self, tokens: list):
        n = len(tokens) // self.page
        return [tuple(tokens[i * self.page:(i + 1) * self.page]) for i in range(n)]

    def match(self, tokens: list) -> list:
        """Longest cached page-aligned prefix of `tokens`: the path's nodes (their pages in order), each referenced
        once more until `release`."""
        node, path = self.root, []
        t = next(self.clock)
        for key in self._chunks(tokens):
            nxt = node.children.get(key)
            if nxt is None:
                break
            nxt.ref += 1
            nxt.last = t
            path.append(nxt)
            node = nxt
        self.lookups += 1
        self.hits += bool(path)
        return path

    def release(self, path: list) -> None:
        for n in path:
            n.ref -= 1

    def insert(self, tokens: list, pages: list) -> list:
        """Donate the pages holding tokens[: len(pages) * 64]; returns the pages the tree did not take (prefix
        already cached by another request: the caller frees them)."""
        node, rejected = self.root, []
        t = next(self.clock)
        for key, pg in zip(self._chunks(tokens), pages):
            nxt = node.children.get(key)
            if nxt is None:
                nxt = _Node(node, key, pg)
                node.children[key] = nxt
                self.held += 1
            elif nxt.page != pg:
                rejected.append(pg)
            nxt.last = t
            node = nxt
        return rejected

    def path(self, tokens: list) -> list:
        """The cached nodes of the page-aligned prefix of `tokens`, in order, without referencing them."""
        node, out = self.root, []
        for key in self._chunks(tokens):
            node = node.children.get(key)
            if node is None:
                break
            out.append(node)
        return out

    def set_state(self, node: _Node, state) -> None:
        """Attach (or, with None, drop) the recurrent state after `node`'s last token."""
        node.state = state
        if state is None:
            self.stateful.discard(node)
        else:
            self.stateful.add(node)

    def states(self) -> list:
        """Every node holding a recurrent state."""
        return list(self.stateful)

    def _leaves(self):
        stack = [self.root]
        while stack:
            n = stack.pop()
            if n is not self.root and not n.children and n.ref == 0:
                yield n
            stack.extend(n.children.values())

    def evict(self, n_pages: int) -> int:
        """Free up to `n_pages` pages from unreferenced leaves, least recently used first."""
        freed = 0
        while freed < n_pages:
            leaves = sorted(self._leaves(), key=lambda n: n.last)
            if not leaves:
                break
            for lf in leaves:
                if freed >= n_pages:
                    break
                del lf.parent.children[lf.key]
                self.stateful.discard(lf)
                self.alloc.release([lf.page])
                self.held -= 1
                freed += 1
        return freed

    def clear(self) -> int:
        return self.evict(1 << 62)
