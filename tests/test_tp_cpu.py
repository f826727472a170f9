"""Tensor parallelism on CPU ranks (gloo): a TP=2 engine must generate exactly what the TP=1 engine generates.

The random init is TP-invariant (canonical weight blocks with per-block seeds), the all-reduces run in fp32 over gloo,
and the greedy token is merged from per-rank vocabulary shards.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_optimizations_b200.config import EngineConfig
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

PROMPTS = [[(13 * i + 7 * j) % 500 + 1 for j in range(30 + 25 * i)] for i in range(3)]


def _engine(tp: int, rank: int) -> Engine:
    from inference_optimizations_b200.parallel import dist as D
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=4, chunked_prefill=48,
                        cuda_graphs=False, tp=tp)
    return Engine(ecfg, max_seq=256, tp_rank=rank, tp=tp,
                  all_reduce=D.host_all_reduce if tp > 1 else None,
                  argmax_merge=D.argmax_merge if tp > 1 else None)


def _worker(rank: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        outs = _engine(2, rank).generate(PROMPTS, SamplingParams(max_new_tokens=5))
        if rank == 0:
            q.put(outs)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp2_matches_tp1():
    ref = _engine(1, 0).generate(PROMPTS, SamplingParams(max_new_tokens=5))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
    assert outs == ref
