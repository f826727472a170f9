"""Failure detection for multi-GPU serving, done on the host.

The reference has no watchdog of its own (an illegal memory access surfaced only through NCCL's watchdog,
`tooling/diagnostics/ima_locator.py:6-9`); its failure handling is fallback-by-design and loud refusal
(`moe-gemm/dp-moe-symmetric-memory/numinous_dp_moe.py:400-428`).  Here:

* every device-side wait in this framework's own kernels (peer flags, mbarriers) is bounded and leaves an error code
  in a status word instead of hanging; `check_status` turns a non-zero word into `DeviceWaitTimeout` between steps;
* `Heartbeat` publishes a per-rank timestamp in the rendezvous store from a background thread; before launching the
  next step's collectives a rank calls `check()`, which raises `PeerFailure` naming ranks whose heartbeat is older
  than the timeout or that never joined -- a rank that died between steps is noticed on the host, before anyone
  enters a collective that would wait for it;
* process groups get a short timeout (`init_group`), so a collective that does start without a peer ends with an
  error rather than blocking.
"""
from __future__ import annotations

import threading
import time
from datetime import timedelta
from typing import Callable, Iterable, Optional

import torch
import torch.distributed as dist

STATUS_NAMES = {1: "producer wait", 2: "MMA wait", 3: "consumer wait", 4: "peer did not arrive", 5: "bad index"}


class PeerFailure(RuntimeError):
    def __init__(self, ranks: list, why: str):
        super().__init__(f"peer rank(s) {ranks} failed: {why}")
        self.ranks = ranks


class DeviceWaitTimeout(RuntimeError):
    pass


def init_group(backend: str, rank: int, world: int, timeout_s: float = 30.0, **kw) -> None:
    """init_process_group with a short timeout (collectives without a peer end in an error, not a hang)."""
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s), **kw)


def check_status(words: Iterable[torch.Tensor]) -> None:
    """Raise if any kernel status word is non-zero (read between steps)."""
    for w in words:
        v = int(w.reshape(-1)[0].item())
        if v:
            raise DeviceWaitTimeout(f"device wait gave up: code {v} ({STATUS_NAMES.get(v, 'unknown')})")


class Heartbeat:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, interval_s: float = 0.25,
                 clock: Callable[[], float] = time.time, prefix: str = "iob/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.interval_s, self.clock, self.prefix = timeout_s, interval_s, clock, prefix
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.t_start = clock()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), repr(self.clock()))

    def start(self) -> "Heartbeat":
        self.beat()

        def run():
            while not self._stop.wait(self.interval_s):
                try:
                    self.beat()
                except Exception:        # store gone: the process is shutting down
                    return
        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        """Stop beating (a rank leaving between steps): peers see it as failed after the timeout."""
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval_s + 1)

    def last_seen(self, r: int) -> Optional[float]:
        k = self._key(r)
        if not self.store.check([k]):
            return None
        return float(self.store.get(k).decode())

    def dead_peers(self) -> tuple[list, list]:
        """(ranks whose heartbeat is stale, ranks that never published one and are past the join timeout)."""
        now = self.clock()
        stale, missing = [], []
        for r in range(self.world):
            if r == self.rank:
                continue
            t = self.last_seen(r)
            if t is None:
                if now - self.t_start > self.timeout_s:
                    missing.append(r)
            elif now - t > self.timeout_s:
                stale.append(r)
        return stale, missing

    def check(self) -> None:
        stale, missing = self.dead_peers()
        if stale:
            raise PeerFailure(stale, f"no heartbeat for more than {self.timeout_s:.1f} s")
        if missing:
            raise PeerFailure(missing, "never joined")

    def wait_all(self, timeout_s: Optional[float] = None) -> None:
        """Block until every rank has published a heartbeat (bounded)."""
        t0 = self.clock()
        limit = self.timeout_s if timeout_s is None else timeout_s
        while True:
            missing = [r for r in range(self.world) if r != self.rank and self.last_seen(r) is None]
            if not missing:
                return
            if self.clock() - t0 > limit:
                raise PeerFailure(missing, "never joined")
            time.sleep(0.02)
