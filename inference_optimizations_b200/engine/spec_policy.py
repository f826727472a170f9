"""Load-adaptive speculative decoding: run speculative steps only while they beat plain decode.

Model (the decision rule of `speculative/adaptive-spec-policy/numinous_spec_policy.py:163,280`: pick the verify
width r that maximises n * E[tokens | r] / t(n, r)):
  * acceptance is geometric with per-draft probability p, fitted to the observed mean number of accepted drafts
    per speculative step: sum_{i=1..k} p^i = accepted;  E[tokens | r rows] = sum_{i=0..r-1} p^i (bonus included).
  * step cost t(r) is measured online (seconds per engine step, exponential moving average) for the two widths this
    engine runs: r = 1 (plain decode) and r = k + 1 (k drafts + the anchor).

A plain decode step stores its target hidden where the next draft extend reads it, which keeps the draft head in sync
only while the extend window (4 positions) has room; so this engine decides per running set: it probes
`probe_steps` speculative steps, prices one plain step once that is harmless, then keeps the better mode until the
set of running requests changes (new arrivals or completions), when it probes again.  Requests whose draft fell out
of sync stay on plain decode.  `mode="always"` keeps speculation on.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional


def geometric_p(accepted: float, k: int) -> float:
    """p with sum_{i=1..k} p^i = accepted (0 <= accepted <= k), by bisection."""
    accepted = min(max(accepted, 0.0), float(k))
    if accepted <= 0.0:
        return 0.0
    if accepted >= k:
        return 1.0
    lo, hi = 0.0, 1.0
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        s = sum(mid ** i for i in range(1, k + 1))
        if s < accepted:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def expected_tokens(p: float, rows: int) -> float:
    """Tokens emitted per step when verifying `rows` rows (the anchor plus rows - 1 drafts)."""
    return sum(p ** i for i in range(rows))


@dataclass
class SpecPolicy:
    draft_tokens: int
    mode: str = "adaptive"           # "adaptive" | "always"
    probe_steps: int = 6
    ema: float = 0.7
    t_spec: Optional[float] = None
    t_plain: Optional[float] = None
    accepted: Optional[float] = None
    spec_seen: int = 0
    decided: Optional[bool] = None   # None while probing
    running_key: Optional[frozenset] = None
    history: list = field(default_factory=list)

    def _avg(self, old: Optional[float], new: float) -> float:
        return new if old is None else self.ema * old + (1.0 - self.ema) * new

    def reset(self) -> None:
        self.t_spec = self.t_plain = self.accepted = None
        self.spec_seen = 0
        self.decided = None

    def use_spec(self, rids, can_spec: bool = True, can_price: bool = True) -> bool:
        """Decide the mode of the next decode step for the running requests `rids`.  `can_spec`: every request's
        draft head is in sync (a speculative step is possible); `can_price`: a plain step would keep it in sync."""
        if not can_spec:
            return False
        if self.mode == "always":
            return True
        key = frozenset(rids)
        if key != self.running_key:
            self.running_key = key
            self.reset()
        if self.decided is not None:
            return self.decided
        if self.spec_seen < self.probe_steps:
            return True
        if self.t_plain is None:
            return not can_price          # one plain step prices the alternative once it is harmless
        self.decided = self.spec_gain() > 1.0
        self.history.append({"accepted": self.accepted, "t_spec": self.t_spec, "t_plain": self.t_plain,
                             "gain": self.spec_gain(), "spec": self.decided})
        return self.decided

    def observe_spec(self, accepted_mean: float, seconds: float) -> None:
        self.spec_seen += 1
        if self.spec_seen == 1:
            return                        # the first step after a switch carries graph/warm-up cost
        self.t_spec = self._avg(self.t_spec, seconds)
        self.accepted = self._avg(self.accepted, accepted_mean)

    def observe_plain(self, seconds: float) -> None:
        self.t_plain = self._avg(self.t_plain, seconds)

    def spec_gain(self) -> float:
        """Expected tokens/s of speculative steps over plain decode (> 1: speculation pays)."""
        if self.t_spec is None or self.t_plain is None or self.accepted is None:
            return 1.0
        p = geometric_p(self.accepted, self.draft_tokens)
        return expected_tokens(p, self.draft_tokens + 1) / self.t_spec * self.t_plain
