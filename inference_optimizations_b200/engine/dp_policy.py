"""Data-parallel-attention scheduling policies (pure host logic; every DP rank or the DP controller evaluates them on
the same gathered numbers, so all ranks take the same decision).

Under DP attention the ranks run every forward in lock-step (the MoE collectives), so a step lasts as long as the
slowest rank's prefill.  Three rules keep the ranks' prefill work even:

* `DPBalancer` -- cache-aware routing of new requests (`scheduler/dp-balance-and-pacing/dp_prefill_balance.py:1-30`):
  cost(r) = pending uncached prefill tokens of rank r (its last load snapshot plus what was routed there since) +
  the tokens request would have to prefill on r (prompt minus the longest prefix r has seen, from chained block
  hashes); argmin, ties to fewer requests then lower rank.  A returning session matches its previous prompt on its
  rank and stays there unless another rank is idle by more than the prefix it would recompute.
* `prefill_budget` -- per-pass prefill token cap from all ranks' backlogs (`numinous_dp_prefill_budget.py:1-30`): with
  two or more ranks holding backlog the cap is the mean (or median) of the backlogs (each capped at the chunk size),
  at least `min_tokens`, rounded up to the page; no cap when it would not bind.  A long prefill is then split across
  passes so the forward length follows the typical rank, not the outlier (chunk boundaries move; results do not).
* `pace_decide` -- park / release / stock for chunked-prefill continuations (`numinous_dp_pace.py:1-30`): park
  (nobody prefills this pass, everyone decodes) when only continuations would prefill, on at most k_max ranks, some
  other rank has decodes waiting, queues are short, and fewer than `steps` parks happened in a row; otherwise, when
  a continuation runs anyway, release queued new work on other ranks to join the same forward.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Optional, Sequence

BLOCK = 256


def block_hashes(tokens: Sequence[int], block: int = BLOCK) -> list:
    """Chained digest per full block: entry i identifies tokens[0 : (i + 1) * block]."""
    out, h = [], b""
    for i in range(len(tokens) // block):
        m = hashlib.blake2b(h, digest_size=16)
        m.update(",".join(map(str, tokens[i * block:(i + 1) * block])).encode())
        h = m.digest()
        out.append(h)
    return out


class PrefixIndex:
    """LRU-bounded set of block digests one rank has seen."""

    def __init__(self, max_entries: int = 1 << 22):
        self.max_entries = max_entries
        self.d: OrderedDict = OrderedDict()

    def match_blocks(self, hashes: list) -> int:
        n = 0
        for h in hashes:
            if h not in self.d:
                break
            self.d.move_to_end(h)
            n += 1
        return n

    def add(self, hashes: list) -> None:
        for h in hashes:
            self.d[h] = True
            self.d.move_to_end(h)
        while len(self.d) > self.max_entries:
            self.d.popitem(last=False)


@dataclass
class _RankState:
    snapshot_uncached: int = 0
    snapshot_t: float = 0.0
    since: list = field(default_factory=list)          # (t, uncached) routed after the snapshot
    requests: int = 0
    index: PrefixIndex = field(default_factory=PrefixIndex)


class DPBalancer:
    def __init__(self, dp: int, block: int = BLOCK, stick_bias: float = 1.0):
        self.dp, self.block, self.stick_bias = dp, block, stick_bias
        self.ranks = [_RankState() for _ in range(dp)]

    def update_load(self, rank: int, waiting_uncached: int, t: float, requests: Optional[int] = None) -> None:
        """A rank's load snapshot taken at time t (requests routed before t are included in it)."""
        r = self.ranks[rank]
        r.snapshot_uncached, r.snapshot_t = int(waiting_uncached), t
        r.since = [(ts, n) for ts, n in r.since if ts > t]
        if requests is not None:
            r.requests = requests

    def _pending(self, r: _RankState) -> int:
        return r.snapshot_uncached + sum(n for _, n in r.since)

    def costs(self, tokens: Sequence[int]) -> list:
        hs = block_hashes(tokens, self.block)
        matched = [r.index.match_blocks(hs) * self.block for r in self.ranks]
        best = max(matched)
        out = []
        for r, m in zip(self.ranks, matched):
            recompute = len(tokens) - m
            if m < best:
                recompute = len(tokens) - best + (best - m) * self.stick_bias
            out.append(self._pending(r) + recompute)
        return out

    def route(self, tokens: Sequence[int], t: float) -> int:
        c = self.costs(tokens)
        rank = min(range(self.dp), key=lambda i: (c[i], self.ranks[i].requests, i))
        return self.pin(tokens, rank, t)

    def pin(self, tokens: Sequence[int], rank: int, t: float) -> int:
        """Account a request the client pinned to `rank` (the balancer's state stays the same on every rank)."""
        r = self.ranks[rank]
        hs = block_hashes(tokens, self.block)
        uncached = len(tokens) - r.index.match_blocks(hs) * self.block
        r.since.append((t, uncached))
        r.requests += 1
        r.index.add(hs)
        return rank


def prefill_budget(backlogs: Sequence[int], chunk: int, min_tokens: int = 2048, mode: str = "mean",
                   page: int = 64) -> int:
    """Per-pass prefill token cap for every rank (0 = no cap)."""
    if chunk <= 0:
        return 0
    active = [min(int(b), chunk) for b in backlogs if int(b) > 0]
    if len(active) < 2:
        return 0
    t = sorted(active)[len(active) // 2] if mode == "median" else -(-sum(active) // len(active))
    t = max(int(min_tokens), int(t))
    if page > 1:
        t = -(-t // page) * page
    return 0 if t >= max(active) else t


def pace_decide(prefillable: Sequence[bool], cont: Sequence[bool], running: Sequence[int], waiting: Sequence[int],
                streak: int, steps: int = 2, k_max: int = 2, q_max: int = 0, peer: bool = True) -> tuple:
    """-> (action in {"park", "release", "stock"}, next streak)."""
    would = [bool(p) or bool(c) for p, c in zip(prefillable, cont)]
    k = sum(would)
    has_cont = any(bool(c) for c in cont)
    new_work = any(bool(p) and not bool(c) for p, c in zip(prefillable, cont))
    idle_decoders = any(int(r) > 0 and not w for r, w in zip(running, would))
    short_queues = max((int(q) for q in waiting), default=0) <= q_max
    if (steps > 0 and has_cont and not new_work and 1 <= k <= k_max and idle_decoders and short_queues
            and streak < steps):
        return "park", streak + 1
    if has_cont and peer:
        return "release", 0
    return "stock", 0


def skew_chunk_cap(own_extend: int, other_extends: Sequence[int], floor: int = 1024, page: int = 64) -> int:
    """Prefill chunk cap for a rank that would extend while others mostly decode
    (`scheduler/dp-balance-and-pacing/pro_skew_budget_hooks.py:1-20`): max(floor, the largest extend on another
    rank), page aligned, never below one page; 0 = no cap (this rank does not extend)."""
    if own_extend <= 0:
        return 0
    cap = max(int(floor), max((int(x) for x in other_extends), default=0))
    cap = max(page, cap // page * page)
    return cap if cap < own_extend else 0


def moe_pad_rows(counts: Sequence[int]) -> list:
    """Rows each EP rank feeds the grouped expert GEMMs when per-rank token counts differ: the global per-rank mean,
    never below the rank's own count (padding rows carry expert id -1 and are never dispatched) -- so every rank
    sizes its token tiles for the load its experts actually receive
    (`moe-gemm/megamoe-tile-balance/deepgemm_megamoe_hooks.py:7-20`)."""
    if not counts:
        return []
    mean = -(-sum(int(c) for c in counts) // len(counts))
    return [max(int(c), mean) for c in counts]
