"""Flagship serving benchmark: the DSA + MoE model (DeepSeek-V3.2 geometry, FP8 128x128 block-scaled weights) served
with data-parallel attention + expert-parallel MoE over N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W]            (N > 1: launched by torch.distributed.run)
    python bench.py --model gemma31b ...                            (the Gemma-class dense GQA model, tensor parallel)
    python bench.py --impl reference ...                            (the reference arm)

Workload (DSA-MoE): 64 sessions over all ranks (64 / N per rank, each rank its own scheduler and pools), uniform
random token ids, 8192-token prompts, up to 1024 output tokens.  Phase 1 prefills every prompt through the engine
(timed on the device, reported as its own fields: prefill tok/s and time to first token).  Phase 2 decodes all
sessions together: W untimed warm-up steps, then K timed steps.  Every MoE layer is the peer-memory expert exchange
(`parallel/ep.py`); the ranks step in lockstep.  Decode steps replay one CUDA graph per rank (one pinned host->device
copy of the step inputs, one device->host read of the sampled tokens).

Printed by rank 0, one JSON line: `value` = output tokens of the K steps / device time of the step computations (the
graph replays; max over ranks); `e2e` = the same through `Engine.step()` including each step's host->device input copy
and device->host result read, timed on the device around the whole loop (max over ranks).  Weights and KV read per step
(tens of GB) are far larger than the 126 MB L2, so no flush is needed between steps.

Depth: `--layers` (default 13 = the 3 dense layers + 10 MoE layers, the deepest stack whose 256 experts per layer fit
one GPU) is the same at every N so the 1/2/4/8 curve measures one model; at 8 GPUs (or with `--full-depth`) the full
61-layer model (it needs the expert memory of 8 GPUs) runs too and is reported as the `full_depth` field, with its
`vs_baseline` against the published 8 x B200 figure.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

# The reference's published final composed DeepSeek V4 Pro recipe, 64 sessions on 8 x B200: 1,813 - 1,996 steady tok/s
# (`evidence/gate/deepseek-v4-pro_standard_B200:8_final_pro_full_20261002-191557.json` in the reference)
BASELINE_TOK_S = 1996.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--model", default="dsa_moe")
    p.add_argument("--sessions", type=int, default=None, help="sessions over all ranks (dsa_moe 64, gemma31b 32)")
    p.add_argument("--ctx", type=int, default=None, help="prompt tokens (dsa_moe 8192, gemma31b 32768)")
    p.add_argument("--max-new", type=int, default=None, help="output tokens (dsa_moe 1024, gemma31b 512)")
    p.add_argument("--layers", type=int, default=None,
                   help="dsa_moe: depth of the scaling-curve model (13); glm5: depth run on every rank (8)")
    p.add_argument("--full-depth", dest="full_depth", action="store_true", default=None,
                   help="dsa_moe: also run the full 61-layer model (default: on at 8 GPUs, the published config)")
    p.add_argument("--no-full-depth", dest="full_depth", action="store_false")
    p.add_argument("--kv", default="nvfp4", choices=["nvfp4", "fp8", "bf16"])
    p.add_argument("--spec", type=int, default=1,
                   help="gemma31b: 1 = speculative decoding, the config's 1-layer draft proposing 3 tokens; 0 = plain")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--tp-form", default="push", choices=["push", "pull", "nvls"],
                   help="gemma31b, tp > 1: fused GEMM -> all-reduce form (push: GEMM epilogue stores to every rank; "
                        "pull: peer-load reduce; nvls: switch-side reduction)")
    p.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                   help="gemma31b tensor-parallel all-reduce: own peer-memory kernel fused with the norms or NCCL")
    a = p.parse_args()
    if a.model == "glm5":              # long-context config: 8 sessions of 204,800 cached tokens per rank
        a.sessions = a.sessions or 8 * int(os.environ.get("WORLD_SIZE", "1"))
        a.ctx = a.ctx or 204800
        a.max_new = a.max_new or 256
        a.layers = a.layers or 8
        return a
    gemma = a.model != "dsa_moe"
    a.sessions = a.sessions or (32 if gemma else 64)
    a.ctx = a.ctx or (32768 if gemma else 8192)
    a.max_new = a.max_new or (512 if gemma else 1024)
    a.layers = a.layers or 13
    return a


def reference_arm(args) -> None:
    # The reference is a collection of SGLang v0.5.20 patches and kernels; it has no installable package and SGLang
    # is not present on this image, so its serving stack cannot run here.
    print(json.dumps({"impl": "reference", "unavailable": "reference is an SGLang patch set with no setup.py/"
                      "pyproject (pip: 'not installable') and SGLang is not installed offline"}))


def _any_rank(flag: bool, dev) -> bool:
    import torch
    import torch.distributed as dist
    if not dist.is_initialized():
        return flag
    t = torch.tensor([int(flag)], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return bool(t.item())


def _gather_floats(vals: list, dev) -> list:
    """Every rank's list (same length on every rank) concatenated, on every rank."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if not dist.is_initialized():
        return t.tolist()
    out = torch.empty(dist.get_world_size() * t.numel(), dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(out, t)
    return out.tolist()


def _sum_ranks(x: int, dev) -> int:
    import torch
    import torch.distributed as dist
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.int64, device=dev)
    dist.all_reduce(t)
    return int(t.item())


def _tokens_check(eng, dev) -> dict:
    """Correctness of the multi-GPU step on the driver's path: the next decode step of every session computed three
    ways from the same state -- the captured graph (the timed path), eager with the peer-memory expert exchange, eager
    with the NCCL baseline exchange -- must give the same greedy tokens on every rank.  Re-running a step rewrites
    the same KV rows, so the check leaves the sessions as they were (nothing is committed to the scheduler)."""
    runner, model = eng.runner, eng.runner.model
    reqs = list(eng.sched.running)
    graphs = runner.ecfg.cuda_graphs
    out_graph = runner.decode(reqs)
    runner.ecfg.cuda_graphs = False
    try:
        out_eager = runner.decode(reqs)
        for ex in model.ep.values():
            ex.use_nccl = True
        out_nccl = runner.decode(reqs)
    finally:
        for ex in model.ep.values():
            ex.use_nccl = False
        runner.ecfg.cuda_graphs = graphs
    same = int(out_graph == out_eager == out_nccl)
    from inference_optimizations_b200.parallel import dist as D
    return {"tokens_match": bool(D.max_over_ranks(float(1 - same)) == 0.0), "sessions_checked": len(reqs),
            "compared": "greedy tokens of one decode step: CUDA graph (timed path) vs eager peer-memory EP vs eager "
                        "NCCL EP (all-gather + all-to-all), every rank"}


def run_dsa(args, info, dev, layers: int, steps: int, warm: int) -> dict:
    """One DSA-MoE serving run (prefill every prompt, then timed decode steps); the measurements as a dict."""
    import torch
    import torch.distributed as dist
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.mla_runner import pool_capacity
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    from inference_optimizations_b200.parallel import dist as D
    from inference_optimizations_b200.utils.clocks import ClockSampler, rejected

    n, rank = info.world, info.rank
    if args.sessions % n:
        raise SystemExit(f"{args.sessions} sessions do not divide over {n} ranks")
    per = args.sessions // n
    cfg = model_config("dsa_moe", num_layers=layers)
    ecfg = EngineConfig(model="dsa_moe", device=str(dev), kv_dtype=args.kv, max_running=per,
                        chunked_prefill=args.ctx, cuda_graphs=not args.no_graphs, graph_batch_sizes=str(per),
                        ep=n, prefix_cache=False)
    assert args.max_new > warm + steps + 4, "sessions must not finish inside the timed steps"
    t_build = time.perf_counter()
    eng = Engine(ecfg, cfg, max_seq=args.ctx + args.max_new + 64, ep_rank=rank,
                 ep_group=dist.group.WORLD if n > 1 else None)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t_build
    pool = pool_capacity(eng.runner)
    g = torch.Generator().manual_seed(1000 + rank)
    reqs = [eng.add_request(torch.randint(1, cfg.vocab, (args.ctx,), generator=g).tolist(),
                            SamplingParams(max_new_tokens=args.max_new)) for _ in range(per)]
    # ---------------------------------------------------------------- phase 1: prefill every prompt
    if n > 1:
        dist.barrier()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ttft = {}
    t0 = time.perf_counter()
    p0.record()
    while _any_rank(eng.sched.prefilling is not None or bool(eng.sched.waiting), dev):
        out = eng.step()
        now = time.perf_counter() - t0
        for rid in out:
            ttft.setdefault(rid, now)
    p1.record()
    torch.cuda.synchronize()
    prefill_ms = D.max_over_ranks(p0.elapsed_time(p1))
    ttfts = sorted(_gather_floats([1e3 * ttft.get(r.rid, float("nan")) for r in reqs], dev))
    # ---------------------------------------------------------------- phase 2: decode every session
    eng.runner.warm_graphs(per)                      # collective under expert parallelism
    for _ in range(warm):
        eng.step()
    bucket = eng.runner._bucket(per)
    launches_per_step = eng.runner.count_step_launches(bucket)
    table0 = eng.runner.kv.table.bytes_synced if hasattr(eng.runner.kv.table, "bytes_synced") else 0
    torch.cuda.synchronize()
    if n > 1:
        dist.barrier()
    clocks = ClockSampler(info.local_rank).start()
    time.sleep(0.3)
    eng.runner.event_log = []
    n_stats = len(eng.stats)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record()
    toks = 0
    for _ in range(steps):
        out = eng.step()
        toks += sum(len(v) for v in out.values())
    ev1.record()
    torch.cuda.synchronize()
    if n > 1:
        dist.barrier()
    ck = clocks.stop()
    kinds = [st.kind for st in eng.stats[n_stats:]]
    graphed = len(eng.runner.event_log)
    dev_ms = D.max_over_ranks(sum(a.elapsed_time(b) for a, b in eng.runner.event_log))
    e2e_ms = D.max_over_ranks(ev0.elapsed_time(ev1))
    toks_all = _sum_ranks(toks, dev)
    status = 0
    if eng.runner.model.ep:
        for ex in eng.runner.model.ep.values():
            status |= int(ex.status.item()) if hasattr(ex, "status") else 0
    for d in (eng.runner.kv.idx_ws, eng.runner.kv.mla_ws):      # indexer / sparse-MLA bounded waits, range checks
        for ws in d.values():
            status |= int(ws.status.item())
    status = int(D.max_over_ranks(float(status)))
    check = _tokens_check(eng, dev) if n > 1 else None
    table1 = eng.runner.kv.table.bytes_synced if hasattr(eng.runner.kv.table, "bytes_synced") else 0
    h2d = 5 * 4 * bucket + (table1 - table0) // max(1, steps)
    mem_gb = D.max_over_ranks(torch.cuda.max_memory_allocated(dev) / 1e9)
    pct = lambda q: ttfts[min(len(ttfts) - 1, int(q * len(ttfts)))]  # noqa: E731
    res = {
        "value": toks_all / (dev_ms / 1e3),
        "ms_per_step": dev_ms / steps,
        "e2e_value": toks_all / (e2e_ms / 1e3),
        "e2e_ms_per_step": e2e_ms / steps,
        "h2d": h2d, "d2h": 4 * bucket,
        "tokens": toks_all, "timed_kinds": {k: kinds.count(k) for k in set(kinds)}, "graph_replays": graphed,
        "launches": launches_per_step * graphed,
        "prefill": {"tokens": args.sessions * args.ctx, "ms": round(prefill_ms, 2),
                    "tok_s": round(args.sessions * args.ctx / (prefill_ms / 1e3), 1),
                    "ttft_ms": {"mean": round(sum(ttfts) / len(ttfts), 1), "p50": round(pct(0.5), 1),
                                "p99": round(pct(0.99), 1), "max": round(ttfts[-1], 1)},
                    "note": "every session's prompt prefilled through Engine.step() (chunks of one prompt per step "
                            "per rank, sessions queued at t = 0), device time max over ranks; TTFT = host time from "
                            "the start of the phase to the step that returned the session's first token"},
        "status": status, "check": check, "max_mem_gb": round(mem_gb, 1), "build_s": round(build_s, 1),
        "kv_pool": pool,
        "clocks": ck, "rejected": rejected(ck),
    }
    eng.runner.graphs.clear()
    del eng
    return res


def bench_dsa(args) -> int:
    """The flagship serving config: DSA + MoE (DeepSeek-V3.2 geometry, FP8 128x128 weights), DP attention + EP over N GPUs."""
    import torch
    from inference_optimizations_b200.parallel import dist as D

    info = D.init("nccl")
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    steps, warm = args.steps, max(3, args.warmup)
    n = info.world
    r = run_dsa(args, info, dev, args.layers, steps, warm)
    full = None
    if args.full_depth is None:          # the published figures are for the 61-layer model on 8 GPUs
        args.full_depth = n == 8 and args.layers < 61
    if args.full_depth:
        torch.cuda.empty_cache()
        try:
            f = run_dsa(args, info, dev, 61, steps, warm)
        except (RuntimeError, torch.OutOfMemoryError) as e:     # the scaling-curve line is still printed
            f = None
            full = {"layers": 61, "error": f"{type(e).__name__}: {str(e)[:300]}"}
    if args.full_depth and f is not None:
        full = {"layers": 61, "value": round(f["value"], 2), "ms_per_step": round(f["ms_per_step"], 4),
                "e2e_value": round(f["e2e_value"], 2), "per_user_tok_s": round(f["value"] / args.sessions, 3),
                "vs_baseline": round(f["value"] / BASELINE_TOK_S, 3), "prefill": f["prefill"],
                "status": f["status"], "correctness": f["check"], "kv_pool_capacity_at_boot": f["kv_pool"],
                "max_mem_gb": f["max_mem_gb"],
                "clocks": {k: f["clocks"].get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    res = {
        "metric": (f"output tok/s: DSA-MoE decode of {args.sessions} sessions after their {args.ctx}-token prompts "
                   f"were prefilled (DP attention + EP over N GPUs, {args.layers} layers)"),
        "value": round(r["value"], 2),
        "unit": "tok/s",
        "n_gpus": n,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": round(r["ms_per_step"], 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8 (E4M3 weights with 128x128 UE8M0 block scales, activations per 1x128; bf16 between layers)",
        "data": (f"synthetic: uniform random token ids, random-init weights of the named architecture truncated to "
                 f"{args.layers} of its 61 layers (3 dense + {args.layers - 3} MoE); every prompt prefilled for real "
                 "(phase timed as `prefill`)"),
        "config": {"model": "DSA+MoE (DeepSeek-V3 class): hidden 7168, MLA 128 heads (kv_lora 512, rope 64, q_lora "
                            "1536), DSA indexer 64x128 top-2048, 256 experts top-8 + 1 shared (FFN 2048), first 3 "
                            "layers dense (FFN 18432), vocab 129280, FP8 128x128 weights",
                   "layers": args.layers, "full_layers": 61, "global_batch": args.sessions, "seq_len": args.ctx,
                   "output_len": args.max_new, "parallelism": f"dp{n}-attention ep{n}", "kv_cache": args.kv,
                   "sessions_per_rank": args.sessions // n, "cuda_graphs": not args.no_graphs,
                   "timed_steps": r["timed_kinds"],
                   "l2": "no flush: every decode step reads the touched experts and the KV (tens of GB), far larger "
                         "than the 126 MB L2"},
        "per_user_tok_s": round(r["value"] / args.sessions, 3),
        "prefill": r["prefill"],
        "clocks": {k: r["clocks"].get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons", "samples")},
        "e2e": {"value": round(r["e2e_value"], 2), "unit": "tok/s", "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": r["d2h"], "api": "Engine.step()",
                "ms_per_step": round(r["e2e_ms_per_step"], 4)},
        "gpu_launches": r["launches"],
        "status": r["status"],
        "correctness": r["check"],
        "kv_pool_capacity_at_boot": r["kv_pool"],
        "max_mem_gb": r["max_mem_gb"],
        "vs_baseline_note": ("the published reference figure (1,813-1,996 steady tok/s at 64 sessions on 8 x B200) is a 61-layer "
                             "number; see full_depth.vs_baseline (--full-depth)"),
        "impl": "ours",
    }
    if full is not None:
        res["full_depth"] = full
    if r["rejected"]:
        res["clocks"]["rejected"] = r["rejected"]
    if info.rank == 0:
        print(json.dumps(res), flush=True)
    if n > 1:
        D.shutdown()
    return 0
def bench_gemma(args) -> int:
    """The Gemma-class serving config: dense GQA model, tensor parallel over the N GPUs, decode throughput over 32
    sessions whose 32k-token prompts are in the paged pool."""
    import torch
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.synthetic import synth_decode_sessions
    from inference_optimizations_b200.parallel import dist as D
    from inference_optimizations_b200.utils.clocks import ClockSampler, rejected

    info = D.init("nccl")
    tp, rank = info.world, info.rank
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = model_config(args.model)
    steps, warm = args.steps, max(3, args.warmup)
    # generation budget: no session may finish inside the timed steps (up to 4 tokens per speculative step, then
    # the decode-only pass)
    max_new = max(args.max_new, 4 * (steps + warm) + 2 * steps + 16)
    ecfg = EngineConfig(model=args.model, device=str(dev), kv_dtype=args.kv, max_running=args.sessions,
                        chunked_prefill=2048, spec=bool(args.spec), cuda_graphs=not args.no_graphs,
                        graph_batch_sizes=str(args.sessions), tp=tp, fused_comm=args.comm == "fused",
                        tp_push=args.tp_form == "push", tp_nvls=args.tp_form == "nvls")
    max_seq = args.ctx + max_new + 64
    eng = Engine(ecfg, cfg, max_seq=max_seq, tp_rank=rank, tp=tp,
                 all_reduce=D.nccl_all_reduce if tp > 1 else None,
                 argmax_merge=D.argmax_merge if tp > 1 else None)
    synth_decode_sessions(eng, args.sessions, args.ctx, max_new, seed=1)
    eng.runner.warm_graphs(args.sessions)
    torch.cuda.synchronize()
    for _ in range(warm):
        eng.step()
    # the adaptive speculation policy probes, prices and decides before the timed steps (all ranks alike)
    extra = 0
    while ecfg.spec and eng.spec_policy.decided is None and extra < 64:
        eng.step()
        extra += 1
    bucket = eng.runner._bucket(args.sessions)
    launches_by_kind = {k: eng.runner.count_step_launches(bucket, k) for k in (("spec", "decode") if ecfg.spec
                                                                                else ("decode",))}
    n_stats = len(eng.stats)
    torch.cuda.synchronize()
    if tp > 1:
        torch.distributed.barrier()
    clocks = ClockSampler(info.local_rank).start()
    time.sleep(0.3)
    eng.runner.event_log = []
    table0 = sum(t.bytes_synced for t in eng.runner.kv.tables.values())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record()
    toks = 0
    for _ in range(steps):
        out = eng.step()
        toks += sum(len(v) for v in out.values())
    ev1.record()
    kinds = [st.kind for st in eng.stats[n_stats:]]
    launches = sum(launches_by_kind.get(k, 0) for k in kinds)
    torch.cuda.synchronize()
    if tp > 1:
        torch.distributed.barrier()
    ck = clocks.stop()
    dev_ms = D.max_over_ranks(sum(a.elapsed_time(b) for a, b in eng.runner.event_log))
    e2e_ms = D.max_over_ranks(ev0.elapsed_time(ev1))
    decode_only = None
    if ecfg.spec:
        # secondary figure: the same sessions advanced by plain greedy decode steps (device time of the step bodies)
        runner = eng.runner
        for _ in range(2):
            out = runner.decode(list(eng.sched.running))
            eng.sched.commit_decode(out)
        runner.event_log = []
        dtoks = 0
        for _ in range(steps):
            out = runner.decode(list(eng.sched.running))
            eng.sched.commit_decode(out)
            dtoks += sum(len(v) for v in out.values())
        torch.cuda.synchronize()
        d_ms = D.max_over_ranks(sum(a.elapsed_time(b) for a, b in runner.event_log))
        decode_only = {"value": round(dtoks / (d_ms / 1e3), 2), "ms_per_step": round(d_ms / steps, 4),
                       "note": "plain greedy decode of the same sessions (no draft/verify)"}
    stage = eng.runner.stage
    h2d = stage.h2d_bytes() + (sum(t.bytes_synced for t in eng.runner.kv.tables.values()) - table0) // steps
    # per-step result reads: 4 B per session for a plain step, 7 int32 per session for a speculative step
    d2h = sum(4 * args.sessions * (7 if k == "spec" else 1) for k in kinds) // max(1, len(kinds))
    value = toks / (dev_ms / 1e3)
    accept = None
    if ecfg.spec:
        acc = [r.accepted / max(1, r.spec_steps) for r in eng.sched.running]
        accept = sum(acc) / max(1, len(acc))
    res = {
        "metric": (f"output tok/s: Gemma-class dense GQA decode of {args.sessions} sessions holding "
                   f"{args.ctx}-token prompts (tensor parallel over N GPUs)"),
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": tp,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": round(dev_ms / steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": ("synthetic: random token ids and random-init weights of the named architecture; each session's "
                 f"{args.ctx}-token prompt is in the paged KV pool as random well-formed {args.kv} rows "
                 "(the prefill compute is not part of the timed decode steps)"),
        "config": {"model": "Dense GQA hd512 (Gemma-class 31B): 60 layers, hidden 5376, 32 q / 16 kv heads, "
                            "head_dim 256 on SWA-1024 layers and 512 on every 6th (global) layer, GeGLU 21504, "
                            "vocab 262144",
                   "global_batch": args.sessions, "seq_len": args.ctx, "parallelism": f"tp{tp}",
                   "kv_cache": args.kv, "tp_comm": (args.tp_form if args.comm == "fused" else "nccl") if tp > 1 else None, "speculative": bool(ecfg.spec), "draft_tokens": ecfg.draft_tokens if ecfg.spec else 0,
                   "accept_per_step": accept,
                   "l2": "no flush: every step reads weights + KV (~170 GB at N=1), far larger than the 126 MB L2"},
        "per_user_tok_s": round(value / args.sessions, 3),
        "clocks": {"sm_mhz": ck.get("sm_mhz"), "sm_max_mhz": ck.get("sm_max_mhz"), "reasons": ck.get("reasons"),
                   "samples": ck.get("samples")},
        "e2e": {"value": round(toks / (e2e_ms / 1e3), 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "api": "Engine.step()"},
        "gpu_launches": launches,
        "impl": "ours",
    }
    if decode_only is not None:
        res["decode_only"] = decode_only
        hist = eng.spec_policy.history[-1] if eng.spec_policy.history else {}
        res["config"]["spec_policy"] = {
            "mode": ecfg.spec_policy, "timed_steps": {k: kinds.count(k) for k in set(kinds)},
            "probe": {k: (round(v, 5) if isinstance(v, float) else v) for k, v in hist.items()}}
        res["config"]["spec_note"] = ("random-init draft head: acceptance is whatever the untrained draft achieves "
                                      "against the random-init target; the adaptive policy (speculate only while "
                                      "n * E[tokens] / t(step) beats plain decode) priced both modes before the "
                                      "timed steps")
    bad = rejected(ck)
    if bad:
        res["clocks"]["rejected"] = bad
    if rank == 0:
        print(json.dumps(res), flush=True)
    if tp > 1:
        eng.runner.graphs.clear()
        D.shutdown()
    return 0




def bench_long(args) -> int:
    """The long-context config (GLM-5-class: sessions holding `ctx` cached tokens, data-parallel attention + EP over
    the launched ranks): per-user decode rate, and the KV-pool capacity at boot for NVFP4 vs FP8 rows, from the DP
    serving benchmark (`engine/dp_serve.py`; the sessions' prompts sit in the pool as rows written by the pool
    writers, the prefill is not run).  One JSON line from rank 0."""
    from inference_optimizations_b200.engine import dp_serve
    for k, v in (("RANK", "0"), ("LOCAL_RANK", "0"), ("WORLD_SIZE", "1"), ("MASTER_ADDR", "127.0.0.1")):
        os.environ.setdefault(k, v)
    if "MASTER_PORT" not in os.environ:
        import socket
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            os.environ["MASTER_PORT"] = str(sk.getsockname()[1])
    dp_serve.main(["--model", "glm5", "--layers", str(args.layers), "--sessions", str(args.sessions),
                   "--ctx", str(args.ctx), "--steps", str(args.steps), "--warmup", str(max(3, args.warmup)),
                   "--kv", args.kv] + (["--no-graphs"] if args.no_graphs else []))
    return 0


def main() -> int:
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            reference_arm(args)
        return 0
    if args.model == "dsa_moe":
        return bench_dsa(args)
    if args.model == "glm5":
        return bench_long(args)
    return bench_gemma(args)


if __name__ == "__main__":
    sys.exit(main())
