"""Data-parallel attention + expert-parallel MoE decode benchmark for the MLA + DSA + MoE family, on sessions whose
prompts are already in the pool: DeepSeek-V3.2 geometry with FP8 experts (`dsa_moe`), or the long-context GLM-5-class
model with NVFP4 experts (`glm5`: 64 sessions x 204,800 cached tokens, per-user decode rate and KV-pool tokens at
boot against an FP8-KV run).  One process per GPU:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P \\
        -m inference_optimizations_b200.engine.dp_serve --model glm5 --layers 8 --sessions 64 --ctx 204800 --kv nvfp4

Each rank holds the replicated attention / router / dense layers, E / N routed experts of every MoE layer and the
shared expert; its own sessions (synthetic prompts already in its paged pool: random well-formed rows written
through the pool writers, so a decode step reads the bytes it would after a real prefill); every MoE layer is the
peer-memory exchange of `parallel/ep.py`.  Timed: `--steps` decode steps of all sessions (CUDA-graph replays unless
`--no-graphs`), CUDA events, max over ranks; printed: one JSON line (rank 0) with the aggregate and per-user output
tok/s, the pool capacity at boot for NVFP4 and FP8 latent rows, the SM clocks sampled during the timed steps and the
kernels' status word.  `--layers` truncates the depth (the full model needs every GPU of the node).
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
    from ..utils.clocks import ClockSampler, rejected
    from .engine import Engine
    from .mla_runner import pool_capacity
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="dsa_moe")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--sessions", type=int, default=64, help="sessions over all ranks")
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--kv", default="nvfp4")
    ap.add_argument("--no-graphs", action="store_true")
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
    warm = max(3, a.warmup)
    ecfg = EngineConfig(model=a.model, device=str(dev), kv_dtype=a.kv, max_running=per, chunked_prefill=2048,
                        cuda_graphs=not a.no_graphs, graph_batch_sizes=str(per), ep=world, prefix_cache=False)
    eng = Engine(ecfg, cfg, max_seq=a.ctx + a.steps + warm + 64, ep_rank=rank,
                 ep_group=dist.group.WORLD if world > 1 else None)
    torch.cuda.synchronize()
    cap = pool_capacity(eng.runner)
    from .synthetic import synth_mla_sessions
    synth_mla_sessions(eng, per, a.ctx, a.steps + warm + 8, seed=1 + rank)
    if not a.no_graphs:
        eng.runner.warm_graphs(per)                  # collective under expert parallelism
    for _ in range(warm):
        eng.step()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler(local).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    toks = 0
    for _ in range(a.steps):
        out = eng.step()
        toks += sum(len(v) for v in out.values())
    e1.record()
    torch.cuda.synchronize()
    ck = clocks.stop()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    tt = torch.tensor([toks], dtype=torch.int64, device=dev)
    dist.all_reduce(tt)
    status = 0
    for ex in (eng.runner.model.ep or {}).values():
        ex.check()
    for d in (eng.runner.kv.idx_ws, eng.runner.kv.mla_ws):      # indexer / sparse-MLA bounded waits, range checks
        for ws in d.values():
            status |= int(ws.status.item())
    st = torch.tensor([status], dtype=torch.int64, device=dev)
    dist.all_reduce(st, op=dist.ReduceOp.MAX)
    mem = torch.tensor([torch.cuda.max_memory_allocated(dev) / 1e9], device=dev)
    dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    if rank == 0:
        sec = ms.item() / 1e3
        rate = tt.item() / sec
        print(json.dumps({"metric": "output tok/s (DP attention + EP MoE, decode)", "value": round(rate, 2),
                          "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": warm,
                          "ms_per_step": round(ms.item() / a.steps, 3), "per_user_tok_s": round(rate / a.sessions, 3),
                          "dtype": f"bf16 activations, {cfg.weight_dtype} projections, {cfg.expert_dtype} experts",
                          "data": "synthetic sessions (prompts' KV rows written through the pool writers; prefill "
                                  "not run), random-init weights",
                          "config": {"model": a.model, "layers": cfg.num_layers, "full_layers": model_config(
                                         a.model).num_layers, "sessions": a.sessions, "ctx": a.ctx,
                                     "kv_cache": a.kv, "parallelism": f"dp{world}-attention ep{world}",
                                     "cuda_graphs": not a.no_graphs, "sessions_per_rank": per},
                          "kv_pool_capacity_at_boot": cap, "status": st.item(), "max_mem_gb": round(mem.item(), 1),
                          "clocks": {k: ck.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons", "samples")},
                          "rejected": rejected(ck)}),
              flush=True)
    eng.runner.graphs.clear()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
