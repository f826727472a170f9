"""Decode-burst admission rule (`--num-continuous-decode-steps` semantics) and its DP-attention form.

Behaviour of the reference's rule (`scheduler/decode-burst/decode_burst.py:7-37`, patches 0001-0005): after a decode
pass, prefill admission is held until `burst` consecutive decode steps have run, only while requests are running, never
while a chunked prefill is mid-way, and never on an idle scheduler.  Under DP attention every rank must take the same
decision from the same gathered facts (skipping the per-pass collective on one rank aborts the group, patch 0003), so
`dp_hold` decides from the all-gathered per-rank rows: hold while any rank with running decodes has a streak below the
burst AND the busiest rank's waiting queue is at most `queue_cap` (patch 0005), bounded by `max_delay_passes`.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence


def hold_prefill(burst: int, streak: int, last_was_extend: Optional[bool], running: bool,
                 running_prefill_only: bool = False, chunked_prefill_pending: bool = False) -> bool:
    """True when this pass should skip prefill admission and let decode take the step."""
    if burst <= 1 or last_was_extend is None or last_was_extend or chunked_prefill_pending:
        return False
    if not running or running_prefill_only:
        return False
    return streak < burst


def next_streak(burst: int, streak: int, prefill_admitted: bool) -> int:
    if burst <= 1:
        return 0
    return 0 if prefill_admitted else streak + 1


@dataclass
class RankFacts:
    """One rank's row of the per-pass all-gather (the prefill-delayer negotiation, extended by the streak)."""
    waiting: int
    running: int
    streak: int
    last_was_extend: int      # 1 / 0 / -1 (unknown)
    chunked_pending: int
    delayed_passes: int

    def as_row(self) -> list:
        return [self.waiting, self.running, self.streak, self.last_was_extend, self.chunked_pending,
                self.delayed_passes]

    @staticmethod
    def from_row(r: Sequence[int]) -> "RankFacts":
        return RankFacts(*[int(x) for x in r])


def dp_hold(rows: Sequence[RankFacts], burst: int, queue_cap: int = 2, max_delay_passes: int = 8) -> bool:
    """Identical on every rank given identical rows."""
    if burst <= 1 or not rows:
        return False
    if any(r.chunked_pending for r in rows):
        return False
    if max(r.delayed_passes for r in rows) >= max_delay_passes:
        return False
    if max(r.waiting for r in rows) > queue_cap:
        return False
    decoding = [r for r in rows if r.running > 0]
    if not decoding:
        return False
    if any(r.last_was_extend == 1 or r.last_was_extend == -1 for r in decoding):
        return False
    return any(r.streak < burst for r in decoding)
