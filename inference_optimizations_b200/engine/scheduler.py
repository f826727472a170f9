"""Continuous-batching scheduler: waiting queue, chunked prefill, running decode set, decode-burst admission.

Policy (one decision per engine step, the SGLang event-loop shape the reference patches, `tooling/diagnostics/
numinous_step_trace.py:1-12`):
  * if a request is part-way through a chunked prefill, its next chunk runs (a chunk is never held, reference
    `scheduler/decode-burst/0002-*.patch`);
  * else, if requests are waiting and memory allows, a prefill batch is formed from the head of the queue up to
    `chunked_prefill` tokens - unless the decode-burst rule holds prefill admission
    (`scheduler/decode-burst/decode_burst.py:7-37`, re-implemented in `burst.py`);
  * else all running requests decode one step (or one speculative step).
Admission reserves KV pages for the whole prompt plus the generation budget, so a running request never stalls on
memory (no retraction path is needed; the reference's retraction-abort fix covers a case that cannot arise here).
"""
from __future__ import annotations

import itertools
from collections import deque
from dataclasses import dataclass, field
from typing import Optional

from .burst import hold_prefill, next_streak


@dataclass
class SamplingParams:
    max_new_tokens: int = 128
    temperature: float = 0.0       # greedy only in this version
    stop_token_ids: tuple = ()
    ignore_eos: bool = True


@dataclass
class Request:
    rid: int
    prompt: list
    params: SamplingParams
    output: list = field(default_factory=list)
    slot: int = -1                 # row in the page tables
    prefilled: int = 0             # prompt tokens already in the KV pool
    kv_len: int = 0                # tokens in the KV pool
    pending: Optional[int] = None  # sampled token not yet in the pool (the next decode input)
    finished: bool = False
    draft_state: dict = field(default_factory=dict)
    accepted: int = 0              # speculative: drafts accepted in total
    spec_steps: int = 0
    cached_tokens: int = 0         # prompt tokens whose KV came from the prefix cache at admission

    @property
    def prompt_len(self) -> int:
        return len(self.prompt)

    def total_len(self) -> int:
        return self.prompt_len + len(self.output)


@dataclass
class Segment:
    req: Request
    start: int
    tokens: list
    logits: bool


@dataclass
class Batch:
    kind: str                      # "prefill" | "decode"
    segments: list


class Scheduler:
    def __init__(self, max_running: int, chunked_prefill: int, decode_burst: int = 1, can_admit=None, on_admit=None):
        self.max_running = max_running
        self.chunk = chunked_prefill
        self.burst = decode_burst
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.prefilling: Optional[Request] = None
        self.streak = 0
        self.last_was_extend: Optional[bool] = None
        self._ids = itertools.count()
        self.can_admit = can_admit or (lambda req: True)
        self.on_admit = on_admit          # runner hook: may reuse cached KV (sets prefilled / kv_len)
        self.free_slots = list(range(max_running - 1, -1, -1))

    def new_request(self, prompt: list, params: SamplingParams) -> Request:
        r = Request(next(self._ids), list(prompt), params)
        self.waiting.append(r)
        return r

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.prefilling)

    def _admit(self) -> Optional[Request]:
        if not self.waiting or not self.free_slots or len(self.running) >= self.max_running:
            return None
        r = self.waiting[0]
        if not self.can_admit(r):
            return None
        self.waiting.popleft()
        r.slot = self.free_slots.pop()
        if self.on_admit is not None:
            self.on_admit(r)
        return r

    def schedule(self, hold: Optional[bool] = None, chunk_cap: int = 0, park: bool = False) -> Optional[Batch]:
        """hold: the decode-burst decision taken elsewhere (data-parallel ranks decide together, `burst.dp_hold`);
        None = this scheduler's own rule.  chunk_cap: prefill tokens this pass may take (0 = the chunk size).
        park: the data-parallel pacing decision to park a continuing chunked prefill for this pass (the running
        requests decode instead; `dp_policy.pace_decide`, bounded by its step count)."""
        if park and self.prefilling is not None and self.running:
            self.streak = next_streak(self.burst, self.streak, False)
            self.last_was_extend = False
            return Batch("decode", [Segment(r, r.kv_len, [r.pending], True) for r in self.running])
        # an unfinished chunked prefill otherwise always continues; admission follows the decode-burst rule
        if self.prefilling is None:
            if hold is None:
                hold = hold_prefill(self.burst, self.streak, self.last_was_extend, bool(self.running))
            if not hold:
                self.prefilling = self._admit()
        if self.prefilling is not None:
            self.streak = next_streak(self.burst, self.streak, True)
            self.last_was_extend = True
            return self._prefill_chunk(chunk_cap)
        if self.running:
            self.streak = next_streak(self.burst, self.streak, False)
            self.last_was_extend = False
            return Batch("decode", [Segment(r, r.kv_len, [r.pending], True) for r in self.running])
        return None

    def facts(self) -> list:
        """This scheduler's row of the data-parallel negotiation (`burst.RankFacts` order) plus its prefill backlog
        (prompt tokens not yet in the pool, the `prefill_budget` input)."""
        ext = -1 if self.last_was_extend is None else int(self.last_was_extend)
        backlog = sum(r.prompt_len - r.prefilled for r in self.waiting)
        if self.prefilling is not None:
            backlog += self.prefilling.prompt_len - self.prefilling.prefilled
        return [len(self.waiting), len(self.running), self.streak, ext, int(self.prefilling is not None), backlog]

    def _prefill_chunk(self, cap: int = 0) -> Batch:
        segs, budget = [], min(self.chunk, cap) if cap > 0 else self.chunk
        while self.prefilling is not None and budget > 0:
            r = self.prefilling
            n = min(budget, r.prompt_len - r.prefilled)
            last = r.prefilled + n == r.prompt_len
            segs.append(Segment(r, r.prefilled, r.prompt[r.prefilled:r.prefilled + n], last))
            r.prefilled += n
            budget -= n
            if not last:
                break
            self.prefilling = self._admit() if budget > 0 else None
        return Batch("prefill", segs)

    def plan_prefill(self) -> Optional[Batch]:
        """The next prefill chunk regardless of the decode-burst rule, or None: the prefill lane of the SM-partitioned
        lanes runs beside decode, so it never holds prefill back."""
        if self.prefilling is None:
            self.prefilling = self._admit()
        return self._prefill_chunk() if self.prefilling is not None else None

    def decode_batch(self) -> Optional[Batch]:
        """Every running request, one decode token each (the decode lane's batch)."""
        if not self.running:
            return None
        return Batch("decode", [Segment(r, r.kv_len, [r.pending], True) for r in self.running])

    def commit_prefill(self, batch: Batch, next_tokens: dict) -> None:
        for s in batch.segments:
            r = s.req
            r.kv_len = s.start + len(s.tokens)
            if s.logits:
                r.pending = next_tokens[r.rid]
                r.output.append(r.pending)
                self.running.append(r)
                self._check_done(r)

    def commit_decode(self, new_tokens: dict) -> None:
        """new_tokens: rid -> list of tokens appended this step (1, or 1 + accepted drafts)."""
        for r in list(self.running):
            toks = new_tokens.get(r.rid)
            if not toks:
                continue
            r.kv_len += len(toks)        # the previous pending token and the accepted drafts are now in the pool
            for t in toks:
                if len(r.output) >= r.params.max_new_tokens:
                    break
                r.output.append(t)
            r.pending = toks[-1]
            self._check_done(r)

    def _check_done(self, r: Request) -> None:
        done = len(r.output) >= r.params.max_new_tokens or (
            not r.params.ignore_eos and r.output and r.output[-1] in r.params.stop_token_ids)
        if done:
            r.finished = True
            if r in self.running:
                self.running.remove(r)
            self.free_slots.append(r.slot)

    def finished_requests(self) -> list:
        return []
