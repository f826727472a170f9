"""Data-parallel attention + expert-parallel MoE on CPU ranks (gloo): each rank serves its own requests, the MoE
layers exchange tokens with the collective EP reference, idle ranks join the exchanges, and the outputs equal a
single-process engine holding every expert.

The random init is EP-invariant (each expert seeded by its own name), so the EP=2 model is the EP=1 model split.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

# rank 0 gets three prompts (one long: chunked prefill over several steps), rank 1 one short prompt -> rank 1 idles
PROMPTS = [[(17 * i + 5 * j) % 500 + 1 for j in range(20 + 45 * i)] for i in range(4)]
SPLIT = {0: [0, 2, 3], 1: [1]}


def _engine(ep: int, rank: int, spec: bool = False, model: str = "tiny_mla") -> Engine:
    # the hybrid model's recurrent prefill rounds differently for other chunk boundaries (and co-batched prompts
    # share a step's chunk budget), so it prefills every prompt in one chunk on both sides of the comparison
    chunk = 512 if model == "tiny_kda" else 32
    ecfg = EngineConfig(model=model, device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=chunk,
                        cuda_graphs=False, ep=ep, prefix_cache=False, spec=spec, spec_policy="always")
    return Engine(ecfg, model_config(model), max_seq=256, ep_rank=rank,
                  ep_group=dist.group.WORLD if ep > 1 else None)


def _worker(rank: int, port: int, spec: bool, q, model: str = "tiny_mla"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        eng = _engine(2, rank, spec, model)
        assert eng.runner.model.layers[-1].ffn["w_gu"].shape[0] == model_config(model).num_experts // 2
        outs = eng.generate_dp([PROMPTS[i] for i in SPLIT[rank]], SamplingParams(max_new_tokens=6))
        q.put((rank, outs))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(spec: bool, model: str = "tiny_mla") -> None:
    ref = _engine(1, 0, spec, model).generate(PROMPTS, SamplingParams(max_new_tokens=6))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, spec, q, model)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for rank, idx in SPLIT.items():
        assert got[rank] == [ref[i] for i in idx], (rank, got[rank], [ref[i] for i in idx])


def test_dp_attention_ep_moe_matches_single_process():
    _run(spec=False)


def test_dp_ep_hybrid_kda_model_matches_single_process():
    """The hybrid KDA + MLA + MoE model under DP attention + EP: each rank's recurrent states stay with its own
    requests while the MoE layers exchange tokens; outputs equal the single-process engine."""
    _run(spec=False, model="tiny_kda")


def test_dp_ep_with_mtp_speculation():
    _run(spec=True)


def _policy_worker(rank: int, port: int, q):
    """generate_dp with the DP policies on: decode burst 3 (joint dp_hold), a prefill budget from the backlogs, and
    cache-aware routing of the global prompt list."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                            cuda_graphs=False, ep=2, prefix_cache=False, decode_burst=3)
        eng = Engine(ecfg, model_config("tiny_mla"), max_seq=256, ep_rank=rank, ep_group=dist.group.WORLD)
        outs = eng.generate_dp(PROMPTS, SamplingParams(max_new_tokens=6), route=True)
        q.put((rank, outs, eng.dp_log))
    finally:
        dist.destroy_process_group()


def test_dp_policies_in_the_serving_loop():
    """Routed prompts are each served once; every rank took the same hold / budget decision every pass; bursts held
    prefill admission on some passes; greedy outputs equal the single-process engine's."""
    ref = _engine(1, 0).generate(PROMPTS, SamplingParams(max_new_tokens=6))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_policy_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, outs, log = q.get(timeout=600)
        got[rank] = (outs, log)
    for p in procs:
        p.join(timeout=120)
    served = {}
    for rank in (0, 1):
        served.update(got[rank][0])
    assert sorted(served) == list(range(len(PROMPTS)))
    assert set(got[0][0]).isdisjoint(got[1][0]) and got[0][0] and got[1][0]
    assert all(served[i] == ref[i] for i in served), (served, ref)
    assert got[0][1] == got[1][1]                     # identical joint decisions on both ranks
    assert any(h for h, *_ in got[0][1])              # decode bursts held prefill on some passes


PACE_SPLIT = {0: [[(3 * j + 1) % 500 + 1 for j in range(20)], [(7 * j + 2) % 500 + 1 for j in range(200)]],
              1: [[(5 * j + 3) % 500 + 1 for j in range(20)], [(11 * j + 4) % 500 + 1 for j in range(30)]]}


def _pace_worker(rank: int, port: int, q):
    """generate_dp with pacing (park a lone continuing chunked prefill for up to 2 passes while the other rank only
    decodes) and the skew chunk cap on."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                            cuda_graphs=False, ep=2, prefix_cache=False, dp_pace_steps=2, dp_skew_floor=64)
        eng = Engine(ecfg, model_config("tiny_mla"), max_seq=256, ep_rank=rank, ep_group=dist.group.WORLD)
        outs = eng.generate_dp(PACE_SPLIT[rank], SamplingParams(max_new_tokens=6))
        q.put((rank, outs, eng.dp_log))
    finally:
        dist.destroy_process_group()


def test_dp_pacing_and_skew_cap_in_the_serving_loop():
    """Pacing parks rank 0's long chunked prefill on some passes (its running request decodes instead) and the
    outputs still equal the single-process engine's: the policies move work between passes, never change it."""
    prompts = PACE_SPLIT[0] + PACE_SPLIT[1]
    ref = _engine(1, 0).generate(prompts, SamplingParams(max_new_tokens=6))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pace_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, outs, log = q.get(timeout=600)
        got[rank] = (outs, log)
    for p in procs:
        p.join(timeout=120)
    assert got[0][0] == ref[:2] and got[1][0] == ref[2:], (got, ref)
    assert [p for *_, p in got[0][1]] == [p for *_, p in got[1][1]]    # one pacing decision per pass, all ranks
    parks = sum(p for *_, p in got[0][1])
    assert 1 <= parks, got[0][1]
