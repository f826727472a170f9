"""Failure detection on the host (parallel/health.py), with failures injected on the host only: a rank that leaves
between steps, a rank that never joins, a rank that raises before a collective, dropped heartbeat messages, and a
device status word carrying a bounded-wait timeout.  Multi-process cases run as gloo ranks on CPU."""
import os
import time

import pytest
import torch
import torch.multiprocessing as mp

from inference_optimizations_b200.parallel import health as HL


class DictStore:
    """In-process stand-in for the rendezvous store; `drop` swallows writes of the given keys (lost messages)."""

    def __init__(self):
        self.d, self.drop = {}, set()

    def set(self, k, v):
        if k not in self.drop:
            self.d[k] = v.encode() if isinstance(v, str) else v

    def get(self, k):
        return self.d[k]

    def check(self, keys):
        return all(k in self.d for k in keys)


class FakeClock:
    def __init__(self):
        self.t = 1000.0

    def __call__(self):
        return self.t


def test_never_joined_and_stale_with_fake_clock():
    st, clk = DictStore(), FakeClock()
    hb0 = HL.Heartbeat(st, 0, 3, timeout_s=5.0, clock=clk)
    hb1 = HL.Heartbeat(st, 1, 3, timeout_s=5.0, clock=clk)
    hb0.beat()
    hb1.beat()
    hb0.check()                                    # rank 2 not yet past the join timeout
    clk.t += 6.0
    hb0.beat()
    with pytest.raises(HL.PeerFailure) as e:
        hb0.check()
    assert e.value.ranks == [1]                    # rank 1 stale (checked before never-joined rank 2)
    hb1.beat()
    with pytest.raises(HL.PeerFailure) as e:
        hb0.check()
    assert e.value.ranks == [2] and "never joined" in str(e.value)


def test_dropped_heartbeats_mark_the_sender_failed():
    st, clk = DictStore(), FakeClock()
    hb0, hb1 = HL.Heartbeat(st, 0, 2, timeout_s=2.0, clock=clk), HL.Heartbeat(st, 1, 2, timeout_s=2.0, clock=clk)
    for _ in range(3):
        hb0.beat(), hb1.beat()
        clk.t += 1.0
        hb0.check()
    st.drop.add("iob/hb/1")                        # rank 1's messages stop arriving
    for _ in range(3):
        hb0.beat(), hb1.beat()
        clk.t += 1.0
    with pytest.raises(HL.PeerFailure):
        hb0.check()


def test_status_word_timeout_is_reported():
    HL.check_status([torch.zeros(1, dtype=torch.int32)])
    with pytest.raises(HL.DeviceWaitTimeout, match="peer did not arrive"):
        HL.check_status([torch.zeros(1, dtype=torch.int32), torch.tensor([4], dtype=torch.int32)])


def _report(q, item):
    q.put(item)
    q.close()
    q.join_thread()                                # flushed before the process ends


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    HL.init_group("gloo", rank, world, timeout_s=4.0)
    store = dist.distributed_c10d._get_default_store()
    hb = HL.Heartbeat(store, rank, world, timeout_s=1.5, interval_s=0.1).start()
    hb.wait_all(10.0)
    x = torch.ones(4)
    try:
        for step in range(6):
            if mode == "leave" and rank == 1 and step == 2:
                hb.stop()                          # leaves between steps: nothing of it is in flight
                _report(q, (rank, "left", step))
                time.sleep(4.0)
                os._exit(0)
            if mode == "raise" and rank == 1 and step == 2:
                raise RuntimeError("injected failure on rank 1")
            if mode == "leave":
                t0 = time.time()
                while True:                        # the host learns of the failure before the next launch
                    hb.check()
                    if time.time() - t0 > 2.0:
                        break
                    time.sleep(0.05)
            dist.all_reduce(x)
        _report(q, (rank, "finished", -1))
    except HL.PeerFailure as e:
        _report(q, (rank, "peer_failure", e.ranks))
    except Exception as e:                         # collective ended with an error instead of blocking
        _report(q, (rank, "collective_error", type(e).__name__))
    os._exit(0)


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() + len(mode)) % 200
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    t0 = time.time()
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, what, info = q.get(timeout=60)
        res[r] = (what, info)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res, time.time() - t0


def test_rank_leaving_between_steps_is_detected_before_the_next_collective():
    res, _ = _run("leave")
    assert res[1] == ("left", 2)
    assert res[0] == ("peer_failure", [1])


def test_rank_raising_ends_the_peers_collective_with_an_error():
    res, dt = _run("raise")
    assert res[0][0] == "collective_error"
    assert dt < 45
