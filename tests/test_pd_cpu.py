"""Prefill / decode disaggregation (engine/pd_serve.py) on two CPU ranks (gloo): rank 0 prefills, rank 1 decodes;
pages are reserved on the decode side before the prompt runs, handed over after it, and the decode rank's outputs
equal one engine's.  On CPU ranks the pages travel in the host messages (the GPU pair copies them over peer memory,
tests/test_pd_gpu.py); the protocol -- reservation, hand-over, first token, decode admission -- is the same."""
import os
import socket

import torch.distributed as dist
import torch.multiprocessing as mp

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

PROMPTS = [[(13 * i + 7 * j) % 500 + 1 for j in range(20 + 41 * i)] for i in range(4)]


def _ecfg(running: int) -> EngineConfig:
    return EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=running, chunked_prefill=48,
                        cuda_graphs=False, prefix_cache=False, max_total_tokens=4096)


def _worker(rank: int, port: int, running: int, q):
    from inference_optimizations_b200.engine.pd_serve import PDPair
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        pair = PDPair(_ecfg(running), model_config("tiny_mla"), max_seq=256, cpu_group=dist.group.WORLD)
        outs = pair.serve(PROMPTS if rank == 1 else None, SamplingParams(max_new_tokens=5))
        q.put((rank, outs, pair.transfers))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_pd_pair_matches_one_engine_cpu():
    running = 2
    ref = Engine(_ecfg(running), model_config("tiny_mla"), max_seq=256).generate(PROMPTS,
                                                                                  SamplingParams(max_new_tokens=5))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, running, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {r: (o, n) for r, o, n in (q.get(timeout=600) for _ in range(2))}
    for p in procs:
        p.join(timeout=120)
    assert got[1][0] == ref, (got[1][0], ref)
    assert got[0][0] == [] and got[0][1] == len(PROMPTS)
