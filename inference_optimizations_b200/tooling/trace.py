"""Per-rank engine step trace (JSONL), the engine-native form of the reference's scheduler trace
(`tooling/diagnostics/sched_trace_hooks.py:1-43,172-306`, `numinous_step_trace.py:1-12`).

One record per engine step: step index, rank, kind (prefill / decode / spec), running / waiting counts, tokens,
host phase times (schedule, run, commit) and the device time of the step body.  The device time comes from CUDA
events that are read only once they have completed (`Event.query()`), so tracing never adds a host sync; records
wait in a small queue until their events are done and are flushed in batches.
"""
from __future__ import annotations

import json
import os
import time
from collections import deque
from typing import Optional

import torch


class StepTrace:
    def __init__(self, directory: str, rank: int = 0, flush_every: float = 0.5):
        os.makedirs(directory, exist_ok=True)
        self.path = os.path.join(directory, f"trace.rank{rank}.jsonl")
        self.rank = rank
        self.flush_every = flush_every
        self.pending: deque = deque()
        self.ready: list = []
        self.last_flush = time.perf_counter()
        self.step = 0

    def begin(self) -> dict:
        rec = {"step": self.step, "rank": self.rank, "t": time.time(), "phases": {}}
        self.step += 1
        return rec

    def phase(self, rec: dict, name: str, t0: float) -> float:
        t1 = time.perf_counter()
        rec["phases"][name] = round((t1 - t0) * 1e3, 4)
        return t1

    def end(self, rec: dict, events: Optional[tuple] = None) -> None:
        self.pending.append((rec, events))
        self._drain()
        if time.perf_counter() - self.last_flush > self.flush_every:
            self.flush()

    def _drain(self) -> None:
        while self.pending:
            rec, ev = self.pending[0]
            if ev is not None:
                if not ev[1].query():
                    break
                rec["gpu_ms"] = round(ev[0].elapsed_time(ev[1]), 4)
            self.ready.append(rec)
            self.pending.popleft()

    def flush(self, wait: bool = False) -> None:
        if wait and torch.cuda.is_available():
            torch.cuda.synchronize()
        self._drain()
        if self.ready:
            with open(self.path, "a") as f:
                for r in self.ready:
                    f.write(json.dumps(r) + "\n")
            self.ready.clear()
        self.last_flush = time.perf_counter()


def read(path: str) -> list:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]
