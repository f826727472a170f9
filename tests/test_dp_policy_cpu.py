"""DP-attention scheduling policies (engine/dp_policy.py): cache-aware routing (sticky sessions, cold prompts spread,
snapshots plus in-flight routing), the per-pass prefill budget, and the park / release pacing rule."""
import random

from inference_optimizations_b200.engine import dp_policy as P


def test_block_hashes_identify_prefixes():
    a = list(range(1000))
    b = a[:512] + [7] * 488
    ha, hb = P.block_hashes(a, 256), P.block_hashes(b, 256)
    assert len(ha) == 3 and ha[:2] == hb[:2] and ha[2] != hb[2]


def test_returning_session_sticks_and_cold_prompts_spread():
    bal = P.DPBalancer(4, block=256)
    rng = random.Random(0)
    sessions = [[rng.randrange(50000) for _ in range(4096)] for _ in range(8)]
    first = [bal.route(s, t=0.0) for s in sessions]
    # 8 cold prompts of equal size spread over the 4 ranks evenly (burst: no snapshot yet)
    assert sorted(first.count(r) for r in range(4)) == [2, 2, 2, 2]
    for r in range(4):
        bal.update_load(r, 0, t=1.0)                  # everything prefilled
    # second turn: previous prompt + new tokens -> same rank (its prefix is cached there)
    for s, r0 in zip(sessions, first):
        turn2 = s + [rng.randrange(50000) for _ in range(300)]
        assert bal.route(turn2, t=2.0) == r0


def test_idle_rank_wins_over_a_short_prefix():
    bal = P.DPBalancer(2, block=256)
    s = list(range(512))
    assert bal.route(s, 0.0) == 0
    bal.update_load(0, 100000, t=1.0)                 # rank 0 is buried in prefill work
    bal.update_load(1, 0, t=1.0)
    assert bal.route(s + list(range(600, 700)), 2.0) == 1


def test_prefill_budget():
    assert P.prefill_budget([0, 16384, 0, 0], 16384) == 0           # one active rank: no cap
    t = P.prefill_budget([16384, 1000, 1200, 0], 16384, min_tokens=2048, page=64)
    assert t == ((16384 + 1000 + 1200) // 3 + 63) // 64 * 64
    assert P.prefill_budget([3000, 3000], 16384) == 0                 # would not bind
    assert P.prefill_budget([16384, 10, 10], 16384, mode="median") == 2048


def test_pace_park_and_release():
    # only rank 0 continues a chunked prefill, rank 1 has decodes: park up to `steps` times, then run it
    args = dict(prefillable=[False, False], cont=[True, False], running=[0, 5], waiting=[0, 0])
    a, s = P.pace_decide(streak=0, **args)
    assert (a, s) == ("park", 1)
    a, s = P.pace_decide(streak=s, **args)
    assert (a, s) == ("park", 2)
    a, s = P.pace_decide(streak=s, **args)
    assert (a, s) == ("release", 0)
    # new work somewhere: never park
    assert P.pace_decide([False, True], [True, False], [0, 5], [0, 1], 0)[0] == "release"
    # nothing continuing: stock
    assert P.pace_decide([True, False], [False, False], [0, 5], [1, 0], 0) == ("stock", 0)


def test_skew_chunk_cap_and_moe_pad_rows():
    assert P.skew_chunk_cap(4096, [0, 1, 1], floor=1024) == 1024
    assert P.skew_chunk_cap(4096, [4096, 0], floor=1024) == 0          # balanced prefills run uncapped
    assert P.skew_chunk_cap(0, [10]) == 0
    assert P.skew_chunk_cap(3000, [2000], floor=512, page=256) == 1792
    assert P.moe_pad_rows([4096, 0, 96, 96]) == [4096, 1072, 1072, 1072]
    assert P.moe_pad_rows([8, 8]) == [8, 8]


def test_router_piggyback_round_trip():
    import torch
    from inference_optimizations_b200.ops import moe as MOE
    sc = torch.rand(5, 56)
    ids = torch.randint(0, 256, (5, 8), dtype=torch.int32)
    w = torch.rand(5, 8)
    packed = MOE.piggyback_pack(sc, ids, w, kmax=9)
    assert packed.shape == (5, 56 + 18)
    s2, i2, w2 = MOE.piggyback_unpack(packed, 56, 9, 8)
    assert torch.equal(s2, sc) and torch.equal(i2, ids) and torch.equal(w2, w)
    assert torch.all(packed[:, 56 + 8] == -1)


def test_scheduler_park_defers_a_continuing_prefill():
    """park=True (the pacing decision): a request part-way through its chunked prefill waits one pass while the
    running requests decode; the next pass resumes the prefill where it stopped."""
    from inference_optimizations_b200.engine.scheduler import SamplingParams, Scheduler
    s = Scheduler(max_running=4, chunked_prefill=16)
    a = s.new_request(list(range(1, 9)), SamplingParams(max_new_tokens=4))
    b = s.new_request(list(range(1, 41)), SamplingParams(max_new_tokens=4))
    first = s.schedule()
    assert first.kind == "prefill" and [len(x.tokens) for x in first.segments] == [8, 8]
    s.commit_prefill(first, {a.rid: 7})
    assert s.prefilling is b and b.prefilled == 8
    parked = s.schedule(park=True)
    assert parked.kind == "decode" and [x.req for x in parked.segments] == [a] and b.prefilled == 8
    s.commit_decode({a.rid: [9]})
    resumed = s.schedule()
    assert resumed.kind == "prefill" and resumed.segments[0].req is b and resumed.segments[0].start == 8
