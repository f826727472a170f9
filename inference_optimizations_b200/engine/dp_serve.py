"""Data-parallel attention + expert-parallel MoE serving benchmark for the MLA + DSA + MoE family (the flagship serving config
shape: DeepSeek-V3.2 geometry, FP8 block-scaled experts, EP over every GPU of the node).  One process per GPU:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P \\
        -m inference_optimizations_b200.engine.dp_serve --layers 8 --sessions 64 --ctx 8192 --steps 20

Each rank holds the replicated attention / router / dense layers, E / N routed experts of every MoE layer and the
shared expert; its own sessions (synthetic prompts already in its paged pool: random well-formed rows); every MoE
layer is the peer-memory exchange of `parallel/ep.py`.  Timed: `--steps` decode steps of all sessions, CUDA events,
max over ranks; printed: one JSON line (rank 0) with the aggregate output tok/s.  `--layers` truncates the depth
(the full 61 layers need every GPU of the node).
"""
from __future__ import annotations

import argparse
import json
import os
from dataclasses import replace

import torch
import torch.distributed as dist


def main(argv=None) -> None:
    from ..config import EngineConfig, model_config
    from .engine import Engine
    from .scheduler import SamplingParams
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="dsa_moe")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--sessions", type=int, default=64, help="sessions over all ranks")
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--kv", default="nvfp4")
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    cfg = model_config(a.model)
    if a.layers:
        cfg = replace(cfg, num_layers=a.layers)
    per = a.sessions // world
    ecfg = EngineConfig(model=a.model, device=str(dev), kv_dtype=a.kv, max_running=per, chunked_prefill=2048,
                        cuda_graphs=False, ep=world, prefix_cache=False)
    eng = Engine(ecfg, cfg, max_seq=a.ctx + a.steps + a.warmup + 64, ep_rank=rank, ep_group=dist.group.WORLD)
    from .synthetic import synth_mla_sessions
    synth_mla_sessions(eng, per, a.ctx, a.steps + a.warmup + 8, seed=1 + rank)
    for _ in range(a.warmup):
        eng.step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    toks = 0
    for _ in range(a.steps):
        out = eng.step()
        toks += sum(len(v) for v in out.values())
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    tt = torch.tensor([toks], dtype=torch.int64, device=dev)
    dist.all_reduce(tt)
    for ex in eng.runner.model.ep.values():
        ex.check()
    if rank == 0:
        sec = ms.item() / 1e3
        print(json.dumps({"metric": "output tok/s (DP attention + EP MoE, decode)", "value": round(tt.item() / sec, 2),
                          "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                          "ms_per_step": round(ms.item() / a.steps, 3), "dtype": "bf16 activations, fp8 experts",
                          "data": "synthetic sessions, random-init weights",
                          "config": {"model": a.model, "layers": cfg.num_layers, "sessions": a.sessions,
                                     "ctx": a.ctx, "kv_cache": a.kv, "parallelism": f"dp{world}-attention ep{world}"}}),
              flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
