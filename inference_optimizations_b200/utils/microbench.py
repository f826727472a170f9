"""Kernel microbenchmarks (CUDA-event timed, warm, inputs larger than L2 unless stated), the small cases the ncu
captures run.  Usage:

    python -m inference_optimizations_b200.utils.microbench gqa_decode --b 8 --ctx 8192 --d 512 --fmt nvfp4
    python -m inference_optimizations_b200.utils.microbench mla_decode --b 64 --heads 128 --ctx 131072 --fmt nvfp4
    python -m inference_optimizations_b200.utils.microbench moe_gemm --b 64 --topk 8 --experts 32 --total-experts 256
    python -m inference_optimizations_b200.utils.microbench hotops --only rmsnorm_fp8,router,kv_write --tokens 64,8192

`--launches N` runs exactly N launches and no timing loop (the form used under ncu: `-s N-1 -c 1`).
Each timed case prints one JSON line with microseconds, bytes moved and GB/s against the measured HBM peak.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

PEAKS = {"hbm_gbs": 6552.0, "bf16_tflops": 1635.7}


def _load_peaks() -> None:
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        PEAKS.update({k: d[k] for k in ("hbm_gbs", "bf16_tflops") if k in d})


def _time(fn, iters: int = 10) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def gqa_decode_case(b: int, hk: int, hq: int, d: int, ctx: int, fmt_name: str, n_q: int, window: int,
                    launches: int = 0, splits_override: str = "", trace: bool = False) -> dict:
    from ..engine.synthetic import fill_pool_random
    from ..ops import attention as A
    from ..ops import kvcache as K
    dev = torch.device("cuda:0")
    fmt = K.FMT_IDS[fmt_name]
    per = (ctx + 63) // 64 + 1
    pages = b * per + 1
    pool = torch.empty(pages, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8, device=dev)
    fill_pool_random(pool, fmt, d, 1)
    pt = (torch.randperm(pages - 1, device=dev)[: b * per] + 1).view(b, per).int()
    kv_len = torch.full((b,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(b * n_q, hq, d, device=dev).to(torch.bfloat16)
    splits = A.split_policy(b * hk, ctx, window)
    if splits_override:                       # "num_splits,tiles_per_split"
        splits = tuple(int(v) for v in splits_override.split(","))
    ws = A.DecodeWorkspace.allocate(b, hk, splits[0], d, device=dev)

    def fn(t=None):
        A.gqa_decode(q, pool, pt, kv_len, n_q, hk, fmt, 1 / math.sqrt(d), window, splits=splits, ws=ws, trace=t)
    if trace:
        # clock64 timeline of CTA 0: event e of tile j at [e * 512 + j] (TraceEv order in attn_gqa_decode.cu);
        # medians over tiles 10 .. n-1 of the per-tile phase lengths
        fn()
        tr = torch.zeros(16 * 512, dtype=torch.int64, device=dev)
        fn(tr)
        torch.cuda.synchronize()
        ev = tr.view(16, 512).cpu()
        n = int((ev[7] > 0).sum())
        med = lambda v: int(v[10:n].median()) if n > 11 else None  # noqa: E731
        return {"kernel": "gqa_decode_trace", "tiles": n, "cycles_per_tile": med(ev[7, 1:n + 1] - ev[7, :n]),
                "k_dequant": med(ev[1] - ev[0]), "v_dequant": med(ev[3] - ev[2]), "qk_issue": med(ev[5] - ev[4]),
                "pv_issue": med(ev[7] - ev[6]), "splits": list(splits)}
    if launches:
        for _ in range(launches):
            fn()
        torch.cuda.synchronize()
        return {}
    us = _time(fn)
    span = min(ctx, window) if window else ctx
    nbytes = b * hk * span * 2 * K.part_bytes(fmt, d) // 64
    return {"kernel": "gqa_decode", "b": b, "hk": hk, "hq": hq, "d": d, "ctx": ctx, "fmt": fmt_name, "n_q": n_q,
            "window": window, "splits": list(splits), "us": round(us, 2), "bytes": nbytes,
            "gbs": round(nbytes / us / 1e3, 1), "frac_hbm": round(nbytes / us / 1e3 / PEAKS["hbm_gbs"], 3)}


def gqa_extend_case(chunk: int, ctx: int, hk: int, hq: int, d: int, fmt_name: str, window: int,
                    launches: int = 0) -> dict:
    """One prefill chunk of `chunk` tokens ending at position ctx (prefix ctx - chunk) through the extend kernel,
    against the same chunk through the decode kernel in n_q-token groups (the prefill path before the extend kernel)."""
    from ..engine.synthetic import fill_pool_random
    from ..ops import attention as A
    from ..ops import kvcache as K
    dev = torch.device("cuda:0")
    fmt = K.FMT_IDS[fmt_name]
    per = (ctx + 63) // 64 + 1
    pool = torch.empty(per + 1, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8, device=dev)
    fill_pool_random(pool, fmt, d, 1)
    pt = (torch.randperm(per, device=dev) + 1).view(1, per).int()
    g = hq // hk
    p0 = ctx - chunk
    q = torch.randn(chunk, hq, d, device=dev).to(torch.bfloat16)
    blocks = torch.tensor(A.extend_blocks([(0, chunk, p0, 0)], g), dtype=torch.int32, device=dev)
    out = torch.zeros_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sm = 1 / math.sqrt(d)

    def fn():
        A.gqa_extend(q, pool, pt, blocks, hk, fmt, sm, window, out=out, status=status)
    if launches:
        for _ in range(launches):
            fn()
        torch.cuda.synchronize()
        return {}
    us = _time_flushed(fn)
    n_q = max(1, 16 // g)
    groups = chunk // n_q
    kvl = (p0 + n_q * torch.arange(1, groups + 1, device=dev)).int()
    rix = torch.zeros(groups, dtype=torch.int32, device=dev)
    splits = (1, 1 << 20)
    ws = A.DecodeWorkspace.allocate(groups, hk, 1, d, device=dev)
    qd = q[: groups * n_q].contiguous()

    def fn_dec():
        A.gqa_decode(qd, pool, pt, kvl, n_q, hk, fmt, sm, window, splits=splits, ws=ws, req_idx=rix)
    us_dec = _time_flushed(fn_dec)
    vis = sum(min(p + 1, window) if window else p + 1 for p in range(p0, ctx))
    flops = 4.0 * hq * d * vis
    peak_f8 = 2 * PEAKS["bf16_tflops"]
    return {"kernel": "gqa_extend", "chunk": chunk, "ctx": ctx, "hk": hk, "hq": hq, "d": d, "fmt": fmt_name,
            "window": window, "blocks": int(blocks.shape[0]), "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1), "frac_f8_peak": round(flops / us / 1e6 / peak_f8, 3),
            "decode_path_us": round(us_dec, 2), "speedup_vs_decode_path": round(us_dec / us, 2)}


def _time_flushed(fn, iters: int = 10) -> float:
    """Mean device time of fn over `iters` launches, L2 flushed before each by READING a 512 MB buffer (a write flush
    would leave ~126 MB of dirty lines whose write-back the timed kernel would pay for), flush not timed."""
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    for _ in range(3):
        fn()
    total = 0.0
    for _ in range(iters):
        torch.sum(flush, dim=0, out=sink)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1)
    return total / iters * 1e3


def mla_pool_random(rows: int, fmt: int, dev, distinct: int = 1 << 16, seed: int = 0) -> torch.Tensor:
    """A pool of `rows` well-formed latent rows (quantized N(0,1) latents), `distinct` unique rows tiled."""
    from ..ops import formats as F
    from ..ops import kvcache as K
    g = torch.Generator(device="cpu").manual_seed(seed)
    n = min(rows, distinct)
    nope = torch.randn(n, F.MLA_NOPE, generator=g)
    rope = torch.randn(n, F.MLA_ROPE, generator=g)
    base = (F.mla_row_quantize(nope, rope) if fmt == K.FMT_NVFP4 else F.mla_fp8_row_quantize(nope, rope)).to(dev)
    reps = -(-rows // n)
    return base.repeat(reps, 1)[:rows].contiguous()


def mla_decode_case(b: int, heads: int, ctx: int, topk: int, fmt_name: str, n_q: int = 1, launches: int = 0,
                    splits_override: str = "") -> dict:
    """The sparse-MLA decode microbenchmark shape: b sequences x n_q query tokens, `heads` heads x 576, `ctx` cached tokens each in a
    page-64 pool, top-`topk` positions per token from a random-normal indexer score, mapped through a random page
    table to pool rows."""
    from ..ops import kvcache as K
    from ..ops import mla as M
    dev = torch.device("cuda:0")
    fmt = K.FMT_IDS[fmt_name]
    per = -(-ctx // 64)
    pages = b * per + 1
    pool = mla_pool_random(pages * 64, fmt, dev)
    pt = (torch.randperm(pages - 1, device=dev)[: b * per] + 1).view(b, per)
    t = b * n_q
    gen = torch.Generator(device=dev).manual_seed(1)
    scores = torch.randn(t, ctx, device=dev, generator=gen)
    pos = scores.topk(topk, dim=-1).indices                                  # [T, topk]
    seq = torch.arange(t, device=dev) // n_q
    idx = (pt[seq[:, None], pos // 64] * 64 + pos % 64).int().contiguous()
    del scores
    q = torch.randn(t, heads, 576, device=dev, generator=gen).to(torch.bfloat16)
    splits = M.mla_split_policy(t, topk)
    if splits_override:                       # "num_splits,tiles_per_split"
        splits = tuple(int(v) for v in splits_override.split(","))
    ws = M.MlaWorkspace.allocate(t, heads, splits[0], device=dev)
    out = torch.empty(t, heads, 512, dtype=torch.bfloat16, device=dev)
    sm = M.mla_sm_scale()

    def fn():
        M.mla_decode(q, pool, idx, sm, fmt, splits=splits, ws=ws, out=out)
    if launches:
        for _ in range(launches):
            fn()
        torch.cuda.synchronize()
        return {}
    us = _time_flushed(fn)
    assert int(ws.status.item()) == 0, "kernel status"
    row_b = M.ROW_BYTES[fmt]
    nbytes = t * topk * row_b + q.numel() * 2 + out.numel() * 2
    flops = 2 * t * heads * topk * (576 + 512)
    return {"kernel": "mla_decode", "tokens": t, "heads": heads, "ctx": ctx, "topk": topk, "fmt": fmt_name,
            "splits": list(splits), "us": round(us, 2), "bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1),
            "tflops": round(flops / us / 1e6, 1),
            "frac_fp8_peak": round(flops / us / 1e6 / (2 * PEAKS["bf16_tflops"]), 3),
            "l2": "flushed before each launch (256 MB write)"}


def indexer_case(b: int, ctx: int, topk: int, heads: int = 64, launches: int = 0) -> dict:
    """DSA indexer at decode: b tokens, each scoring `ctx` cached positions (132 B each) and keeping the top-k."""
    from ..ops import indexer as I
    from ..ops import kvcache as K
    dev = torch.device("cuda:0")
    per = -(-ctx // 64)
    pages = b * per + 1
    pool = torch.randint(0, 256, (pages, K.INDEX_PAGE_BYTES), dtype=torch.uint8, device=dev)
    sc = pool[:, 64 * 128:].view(pages, 64 * 4).view(torch.float32)
    sc.copy_(torch.rand_like(sc) + 0.5)                                  # finite positive key scales
    vals = pool[:, :64 * 128]
    vals[(vals & 0x7F) == 0x7F] = 0                                      # no E4M3 NaN codes
    pt = (torch.randperm(pages - 1, device=dev)[: b * per] + 1).view(b, per).int()
    q8, w = I.indexer_q_quant(torch.randn(b, heads, 128, device=dev), torch.rand(b, heads, device=dev))
    limit = torch.full((b,), ctx, dtype=torch.int32, device=dev)
    ws = I.IndexerWorkspace.allocate(b, ctx, dev)

    def fn():
        I.indexer_select(q8, w, pool, pt, limit, topk, ctx, ws=ws)
    if launches:
        for _ in range(launches):
            fn()
        torch.cuda.synchronize()
        return {}
    us = _time_flushed(fn)
    nbytes = b * ctx * 132
    return {"kernel": "indexer_logits+topk", "tokens": b, "ctx": ctx, "topk": topk, "heads": heads,
            "us": round(us, 2), "bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1),
            "frac_hbm": round(nbytes / us / 1e3 / PEAKS["hbm_gbs"], 3), "l2": "flushed before each launch",
            "kernels_us": _kernel_times(fn)}


def hotops_case(op: str, t: int, hidden: int = 7168, experts: int = 256, launches: int = 0) -> dict:
    """The small per-layer kernels of the DSA-MoE step at `t` tokens:
    `rmsnorm_fp8`  residual add + RMSNorm + E4M3 / UE8M0-per-128 quantization of [t, hidden] (K12/K34 form);
    `router`       sigmoid + bias, group-limited top-8 over fp32 [t, experts] logits, renormalised (K39);
    `kv_write`     NVFP4 352-byte latent rows (512 E2M1 + E4M3 per 16, E4M3 rope) written to t random pool slots (K25).
    Bytes are the op's algorithmic reads + writes; L2 flushed before each launch."""
    from ..ops import basic as B
    from ..ops import kvcache as K
    from ..ops import moe as MOE
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(3)
    if op == "rmsnorm_fp8":
        x = torch.randn(t, hidden, device=dev, generator=g).to(torch.bfloat16)
        res = torch.randn(t, hidden, device=dev, generator=g).to(torch.bfloat16)
        w = torch.rand(hidden, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty_like(x)
        q8 = torch.empty(t, hidden, dtype=torch.uint8, device=dev)
        qs = torch.empty(t, hidden // 128, dtype=torch.int32, device=dev)
        fn = lambda: B.rmsnorm(x, w, 1e-6, residual=res, out=out, fp8=(q8, qs))  # noqa: E731
        nbytes = t * hidden * (2 + 2 + 2 + 2 + 1) + t * hidden // 128 * 4
    elif op == "router":
        logits = torch.randn(t, experts, device=dev, generator=g)
        bias = 0.01 * torch.randn(experts, device=dev, generator=g)
        fn = lambda: MOE.route(logits, bias, 8, 8, 4, 2.5, "sigmoid")  # noqa: E731
        nbytes = t * experts * 4 + t * 8 * 8
    elif op == "kv_write":
        rows = max(1 << 20, 4 * t)
        pool = torch.zeros(rows, 352, dtype=torch.uint8, device=dev)
        nope = torch.randn(t, 512, device=dev, generator=g).to(torch.bfloat16)
        rope = torch.randn(t, 64, device=dev, generator=g).to(torch.bfloat16)
        slot = torch.randperm(rows, device=dev)[:t].int()
        fn = lambda: K.mla_write(nope, rope, slot, pool)  # noqa: E731
        nbytes = t * (576 * 2 + 352 + 4)
    else:
        raise SystemExit(f"hotops: unknown op {op}")
    if launches:
        for _ in range(launches):
            fn()
        torch.cuda.synchronize()
        return {}
    us = _time_flushed(fn, iters=20)
    return {"kernel": op, "tokens": t, "us": round(us, 2), "bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1),
            "frac_hbm": round(nbytes / us / 1e3 / PEAKS["hbm_gbs"], 3), "l2": "flushed before each launch"}


def moe_gemm_case(b: int, experts: int, total_experts: int, topk: int, hidden: int, ffn: int, wfmt: str = "fp8",
                  launches: int = 0) -> dict:
    """Grouped block-scaled expert GEMMs at decode: b tokens routed top-k over `total_experts`; this GPU owns
    experts [0, experts) (the expert-parallel slice).  Weights are random packed blocks (no NaN codes); gate/up
    (fused SwiGLU + requant) and down (routing-weighted bf16 rows) are timed separately.  wfmt: fp8 | nvfp4."""
    from .._ext import ext
    from ..ops import moe_gemm as MG
    dev = torch.device("cuda:0")
    E, H, F = experts, hidden, ffn
    kind = 0 if wfmt == "fp8" else 1
    sfw = 1 if kind == 0 else 4
    vals = 128 if kind == 0 else 256                                      # K values per 128-byte chunk

    def rand_pack(n_tiles, kc, g):
        blk = g * (16384 + 512 * sfw)
        w = torch.randint(0, 256, (E, n_tiles, kc, blk), dtype=torch.uint8, device=dev)
        if kind == 0:
            w[(w & 0x7F) == 0x7F] = 0
        w[..., g * 16384:] = 120 if kind == 0 else 0x30                   # 2^-7 (UE8M0) / 0.5 (E4M3)
        return w
    gd = 2 if (H % 256 == 0 and kind == 0) else 1
    w1, w2 = rand_pack(F // 128, H // vals, 2), rand_pack(H // (128 * gd), F // vals, gd)
    ids = torch.rand(b, total_experts, device=dev).topk(topk, dim=-1).indices.int()
    wts = torch.softmax(torch.randn(b, topk, device=dev), -1)
    x = torch.randn(b, H, device=dev)
    xq, xs = MG.quant_rows(x) if kind == 0 else MG.quant_nvfp4_rows(x)
    P = b * topk
    off = torch.empty(E + 1, dtype=torch.int32, device=dev)
    pairs = torch.empty(P, dtype=torch.int32, device=dev)
    ext().moe_align(ids.view(-1), 0, E, 0, off, pairs)
    local = ids[ids < E]
    n_pairs, touched = int(local.numel()), int(torch.unique(local).numel())
    nt = MG.pick_nt(max(1, -(-2 * n_pairs // E)))
    h = torch.empty(P, F if kind == 0 else F // 2, dtype=torch.uint8, device=dev)
    hs = torch.empty(P, F // 128 if kind == 0 else F // 64, dtype=torch.int32, device=dev)
    rows = torch.empty(P, H, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count

    def gemm1():
        MG.gemm(w1, xq, xs, off, pairs, h, status, n_tiles=F // 128, kc=H // vals, g=2, nt=nt, mode=1, src_div=topk,
                src_limit=P, out_scale=hs, num_ctas=sms, kind=kind)

    def gemm2():
        MG.gemm(w2, h, hs, off, pairs, rows, status, n_tiles=H // (128 * gd), kc=F // vals, g=gd, nt=nt, mode=2,
                src_div=1, pair_w=wts.view(-1), num_ctas=sms, kind=kind)
    if launches:
        for _ in range(launches):
            gemm1()
            gemm2()
        torch.cuda.synchronize()
        return {}
    us1, us2 = _time(gemm1), _time(gemm2)
    torch.cuda.synchronize()
    assert status.item() == 0, status.item()
    wb = 1.0 if kind == 0 else 0.5                                        # weight bytes per value
    sb = (1 / 32) if kind == 0 else (1 / 8)                               # scale-atom bytes per weight byte
    b1 = touched * 2 * F * H * wb * (1 + sb) + n_pairs * (H + F) * wb
    b2 = touched * H * F * wb * (1 + sb) + n_pairs * (F * wb + 2 * H)
    frac = lambda nb, us: round(nb / us / 1e3 / PEAKS["hbm_gbs"], 3)  # noqa: E731
    return {"kernel": f"moe_gemm_{wfmt}_blockscaled", "tokens": b, "topk": topk, "experts_local": E,
            "experts_total": total_experts, "pairs_local": n_pairs, "experts_touched": touched, "nt": nt,
            "hidden": H, "ffn": F, "gate_up_us": round(us1, 2), "gate_up_frac_hbm": frac(b1, us1),
            "down_us": round(us2, 2), "down_frac_hbm": frac(b2, us2), "bytes": int(b1 + b2),
            "l2": "weights per launch exceed L2 (each touched expert read once)"}


def ep_moe_case(tokens: int, total_experts: int, topk: int, hidden: int, ffn: int, wfmt: str = "fp8",
                iters: int = 20) -> dict:
    """Expert-parallel MoE layer (parallel/ep.py) under torchrun: each rank routes `tokens` tokens top-k over
    `total_experts`, owns total_experts / world of them (+ a shared expert); one forward = quantize, dispatch,
    barrier, align, two grouped GEMMs (peer-store epilogue), barrier, combine.  Device time per layer, max over
    ranks (CUDA events around `iters` forwards, synchronized and barriered on both sides); the same for the NCCL
    baseline exchange (`EPMoE.forward_nccl`: all-gather + the same GEMMs + all-to-all) on the same inputs."""
    import torch.distributed as dist
    from ..ops import moe_gemm as MG
    from ..parallel.ep import EPMoE
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    E_loc = total_experts // world
    ex = MG.BlockScaledExperts.random_packed(E_loc, ffn, hidden, wfmt, shared=True, device=dev, seed=rank)
    ep = EPMoE(rank, world, total_experts, tokens, topk, experts=ex)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(tokens, hidden, device=dev, generator=g).to(torch.bfloat16)
    ids = torch.rand(tokens, total_experts, device=dev, generator=g).topk(topk, dim=-1).indices.int()
    w = torch.softmax(torch.randn(tokens, topk, device=dev, generator=g), -1)
    for _ in range(3):
        ep.forward(x, ids, w)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        ep.forward(x, ids, w)
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    ep.check()
    us = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device=dev)
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    # the NCCL baseline exchange (all-gather + all-to-all) around the same GEMMs, same inputs
    ep.use_nccl = True
    for _ in range(3):
        ep.forward(x, ids, w)
    torch.cuda.synchronize()
    dist.barrier()
    e0.record()
    for _ in range(iters):
        ep.forward(x, ids, w)
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    ep.use_nccl = False
    us_nccl = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device=dev)
    dist.all_reduce(us_nccl, op=dist.ReduceOp.MAX)
    # roofline: touched local experts' weights once (HBM) vs rows crossing NVLink
    all_ids = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(all_ids, ids)
    gids = torch.cat(all_ids).view(-1)
    local = gids[(gids >= rank * E_loc) & (gids < (rank + 1) * E_loc)]
    touched = int(torch.unique(local).numel()) + 1                                     # + shared expert
    wb = (1.0 if wfmt == "fp8" else 0.5) * (1 + (1 / 32 if wfmt == "fp8" else 1 / 8))
    w_bytes = touched * 3 * hidden * ffn * wb
    row = hidden * (1.0 if wfmt == "fp8" else 0.5)
    nv_bytes = tokens * topk * (row + 2 * hidden) * (world - 1) / world                  # out + back, remote share
    t_hbm = w_bytes / (PEAKS["hbm_gbs"] * 1e3)
    t_nvl = nv_bytes / (770.0 * 1e3)
    floor = max(t_hbm, t_nvl)
    res = {"kernel": "ep_moe_layer", "fmt": wfmt, "world": world, "tokens_per_rank": tokens, "topk": topk,
           "experts_total": total_experts, "hidden": hidden, "ffn": ffn, "us_max_over_ranks": round(float(us), 1),
           "touched_local_experts": touched, "roofline_us": round(floor, 1),
           "frac_of_roofline": round(floor / float(us), 3),
           "nccl_baseline_us": round(float(us_nccl), 1), "speedup_vs_nccl": round(float(us_nccl) / float(us), 2),
           "roofline_basis": "max(touched weights / measured HBM, remote rows / 770 GB/s)"}
    del ep
    return res if rank == 0 else {}


def tp_gemm_ar_case(tokens: list, K: int, N: int, reps: int = 10, iters: int = 20) -> list:
    """Row-parallel projection + all-reduce + the Gemma norm chain under torchrun (one rank per GPU), three ways:
    `push` -- this framework's GEMM stores its tiles into every rank's slot, then the slot-sum + norm kernel (the
    fused GEMM -> all-reduce); `pull` -- the same GEMM into the own buffer, then the peer-load reduce + norm kernel;
    `nccl` -- the same GEMM, NCCL all-reduce, two RMSNorm kernels; `nvls` (where the buffer has an NVLink multicast
    mapping) -- the same GEMM, then the switch-side reduce + norm kernel.  Each variant is `reps` layers captured in one CUDA
    graph, cycling over enough weight copies that the weights stream from HBM (> 2x L2); device time per layer, max
    over ranks.  Roofline per layer: max(weight bytes / measured HBM, partial rows crossing NVLink / 770 GB/s)."""
    import torch.distributed as dist
    from ..ops import basic as B
    from ..ops import linear as L
    from ..parallel.symm import TPComm
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    n_w = max(2, -(-(256 << 20) // (N * K * 2)))
    lins = [L.Linear((torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16), "bf16")
            for _ in range(n_w)]
    tmax = max(tokens)
    cp = TPComm(rank, world, tmax, N, dev, push=True)
    cq = TPComm(rank, world, tmax, N, dev, push=False)
    try:
        cn = TPComm(rank, world, tmax, N, dev, nvls=True)
    except RuntimeError:
        cn = None
    have = torch.tensor([0.0 if cn is None else 1.0], device=dev)
    dist.all_reduce(have, op=dist.ReduceOp.MIN)          # every rank runs the same variants
    if have.item() == 0:
        cn = None
    w1 = (torch.randn(N, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    w2 = (torch.randn(N, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    rows = []
    for t in tokens:
        x = torch.randn(t, K, device=dev, generator=g).to(torch.bfloat16)
        resid = torch.randn(t, N, device=dev, generator=g).to(torch.bfloat16)

        def push():
            for r in range(reps):
                lins[r % n_w](x, push=cp)
                cp.reduce_norm2(t, resid, w1, w2, 1e-6)

        def pull():
            for r in range(reps):
                lins[r % n_w].lin(x, out=cq.out_buffer(t))
                cq.reduce_norm2(t, resid, w1, w2, 1e-6)

        def nvls():
            for r in range(reps):
                lins[r % n_w].lin(x, out=cn.out_buffer(t))
                cn.reduce_norm2(t, resid, w1, w2, 1e-6)

        def nccl():
            for r in range(reps):
                y = lins[r % n_w](x)
                dist.all_reduce(y)
                o = B.rmsnorm(y, w1, 1e-6, True)
                B.rmsnorm(o, w2, 1e-6, True, residual=resid)

        row = {"kernel": "tp_gemm_ar", "world": world, "tokens": t, "K": K, "N": N}
        variants = [("push", push), ("pull", pull), ("nccl", nccl)] + ([("nvls", nvls)] if cn is not None else [])
        for name, fn in variants:
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            dist.barrier()
            us = torch.tensor([e0.elapsed_time(e1) * 1e3 / (iters * reps)], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            row[f"{name}_us"] = round(float(us), 2)
            del gr
        cp.check()
        cq.check()
        if cn is not None:
            cn.check()
        t_hbm = N * K * 2 / (PEAKS["hbm_gbs"] * 1e3)
        t_nvl = (world - 1) * t * N * 2 / (770.0 * 1e3)
        row.update(roofline_us=round(max(t_hbm, t_nvl), 2), hbm_us=round(t_hbm, 2), nvlink_us=round(t_nvl, 2),
                   push_frac_of_roofline=round(max(t_hbm, t_nvl) / row["push_us"], 3),
                   roofline_basis="max(weights / measured HBM, (world-1) x partial rows / 770 GB/s)")
        rows.append(row)
    torch.cuda.synchronize()
    dist.barrier()
    return rows if rank == 0 else []


def moe_tactics_case(experts: int, total_experts: int, topk: int, hidden: int, ffn: int, wfmt: str) -> dict:
    """Sweep the token tile (MMA N) of the grouped GEMMs over decode / prefill token counts; the fastest per count
    (gate_up + down device time) forms the tactic table `ops/moe_tactics.json`."""
    from .._ext import ext
    from ..ops import moe_gemm as MG
    dev = torch.device("cuda:0")
    E, H, F = experts, hidden, ffn
    kind = 0 if wfmt == "fp8" else 1
    ex = MG.BlockScaledExperts.random_packed(E, F, H, wfmt, shared=False, device=dev)
    vals = 128 if kind == 0 else 256
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    best, raw = {}, {}
    for b in (1, 4, 8, 16, 32, 64, 128, 256, 512, 1024):
        ids = torch.rand(b, total_experts, device=dev).topk(topk, dim=-1).indices.int()
        x = torch.randn(b, H, device=dev)
        xq, xs = MG.quant_rows(x) if kind == 0 else MG.quant_nvfp4_rows(x)
        P = b * topk
        off = torch.empty(E + 1, dtype=torch.int32, device=dev)
        pairs = torch.empty(P, dtype=torch.int32, device=dev)
        ext().moe_align(ids.view(-1), 0, E, 0, off, pairs)
        h = torch.empty(P, F if kind == 0 else F // 2, dtype=torch.uint8, device=dev)
        hs = torch.empty(P, F // 128 if kind == 0 else F // 64, dtype=torch.int32, device=dev)
        rows = torch.empty(P, H, dtype=torch.bfloat16, device=dev)
        w = torch.ones(P, device=dev)
        times = {}
        for nt in (16, 32, 64, 128):
            def run():
                MG.gemm(ex.w1, xq, xs, off, pairs, h, status, n_tiles=F // 128, kc=H // vals, g=2, nt=nt, mode=1,
                        src_div=topk, src_limit=P, out_scale=hs, num_ctas=sms, kind=kind)
                MG.gemm(ex.w2, h, hs, off, pairs, rows, status, n_tiles=H // (128 * ex.g2), kc=F // vals, g=ex.g2,
                        nt=nt, mode=2, src_div=1, pair_w=w, num_ctas=sms, kind=kind)
            times[nt] = round(_time(run), 1)
        raw[b] = times
        best[str(b)] = min(times, key=times.get)
    return {"kernel": "moe_tactics", "fmt": wfmt, "experts_local": E, "experts_total": total_experts,
            "table": {wfmt: best}, "us": raw}


def dense_linear_case(t: int, launches: int = 0) -> dict:
    """Decode-size dense bf16 linears of the flagship model (Gemma-class 31B, TP1): the weight-streaming tcgen05
    GEMM (ops/linear.py) against cuBLAS (torch.nn.functional.linear) on the same tensors, L2 flushed before each
    launch."""
    import torch.nn.functional as Fn
    from ..ops.linear import DenseLinear
    dev = torch.device("cuda:0")
    shapes = {"qkv_swa": (16384, 5376), "o_swa": (5376, 8192), "gate_up": (43008, 5376), "down": (5376, 21504),
              "qkv_global": (32768, 5376), "o_global": (5376, 16384), "lm_head": (262144, 5376)}
    out = {"kernel": "dense_bf16_linear", "tokens": t, "l2": "flushed before each launch", "shapes": {}}
    for name, (n, k) in shapes.items():
        w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
        x = torch.randn(t, k, device=dev).to(torch.bfloat16)
        lin = DenseLinear(w)
        y = torch.empty(t, n, dtype=torch.bfloat16, device=dev)
        if launches:
            for _ in range(launches):
                lin(x, y)
            torch.cuda.synchronize()
            return {}
        ours = _time_flushed(lambda: lin(x, y))
        cub = _time_flushed(lambda: Fn.linear(x, w))
        nb = n * k * 2
        err = float(((lin(x) .float() - Fn.linear(x, w).float()).abs().max()))
        out["shapes"][name] = {"n": n, "k": k, "ours_us": round(ours, 1), "cublas_us": round(cub, 1),
                               "ours_frac_hbm": round(nb / ours / 1e3 / PEAKS["hbm_gbs"], 3),
                               "cublas_frac_hbm": round(nb / cub / 1e3 / PEAKS["hbm_gbs"], 3), "max_abs_diff": err}
        del w, lin
    return out


def proj_gemms_case(tokens: list, only: str = "") -> list:
    """The MLA projection GEMMs of the DSA-MoE layer on the tcgen05 kernels (`ops/linear.py`), each timed alone with
    CUDA events (L2 flushed before each launch): FP8 fused a/b projections, W_o and the LM head, the head-batched bf16
    absorption products, the fp32 router logits.  Reported with the weight-stream bandwidth and the tensor rate."""
    from ..ops import linear as L
    dev = torch.device("cuda:0")
    H, ql, nh = 7168, 1536, 128
    w = lambda n, k: (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    mods = {"a_fp8": (L.Linear(w(2304, H), "fp8"), H, 2304, 1),
            "b_fp8": (L.Linear(w(32768, ql), "fp8"), ql, 32768, 1),
            "o_fp8": (L.Linear(w(H, nh * 128), "fp8"), nh * 128, H, 1),
            "head_fp8": (L.Linear(w(129280, H), "fp8"), H, 129280, 1),
            "router_bf16_f32out": (L.Linear(w(256, H), "bf16"), H, 256, 2),
            "uk_bf16": (L.HeadBatchedLinear((torch.randn(nh, 512, 128, device=dev) * 0.05).to(torch.bfloat16)),
                        128, 512, 2),
            "uv_bf16": (L.HeadBatchedLinear((torch.randn(nh, 128, 512, device=dev) * 0.05).to(torch.bfloat16)),
                        512, 128, 2)}
    out = []
    for t in tokens:
        for name, (m, K, N, wb) in mods.items():
            if (name == "head_fp8" and t > 512) or (only and name not in only.split(",")):
                continue
            if name.startswith("uk"):
                x = torch.randn(t, 256 * 128, device=dev).to(torch.bfloat16)
                fn = lambda m=m, x=x: m(x, t, row_stride=256)  # noqa: E731
                flops, wbytes = 2 * t * nh * K * N, nh * K * N * wb
            elif name.startswith("uv"):
                x = torch.randn(t, nh, 512, device=dev).to(torch.bfloat16)
                fn = lambda m=m, x=x: m(x, t)  # noqa: E731
                flops, wbytes = 2 * t * nh * K * N, nh * K * N * wb
            else:
                x = torch.randn(t, K, device=dev).to(torch.bfloat16)
                f32 = name.startswith("router")
                fn = lambda m=m, x=x, f32=f32: m(x, out_f32=f32) if f32 else m(x)  # noqa: E731
                flops, wbytes = 2 * t * K * N, K * N * wb
            us = _time_flushed(fn)
            row = {"op": name, "tokens": t, "us": round(us, 1), "weight_tb_s": round(wbytes / us / 1e6, 3),
                   "frac_hbm": round(wbytes / us / 1e3 / PEAKS["hbm_gbs"], 3), "tflops": round(flops / us / 1e6, 1)}
            row["kernels_us"] = _kernel_times(fn)
            row["trace_cycles"] = _gemm_trace(fn)
            gemm = sum(v for k, v in row["kernels_us"].items() if "moe_gemm" in k)
            if gemm:
                row["gemm_kernel_frac_hbm"] = round(wbytes / gemm / 1e3 / PEAKS["hbm_gbs"], 3)
            out.append(row)
    return out


def dense_gemms_case(tokens: list, only: str = "") -> list:
    """The Gemma-class (31B) dense projections at one GPU's full width, bf16: this framework's weight-streaming GEMM
    (`ops/linear.py Linear`, split-K by `split_k`) against cuBLAS (`torch.nn.functional.linear`) on the same weights,
    each call timed alone with CUDA events and the L2 flushed before it."""
    import torch.nn.functional as Fn
    from ..ops import linear as L
    from ..ops import moe_gemm as MG
    dev = torch.device("cuda:0")
    h = 5376
    shapes = {"qkv_swa": (16384, h), "qkv_global": (32768, h), "o_swa": (h, 8192), "o_global": (h, 16384),
              "gate_up": (43008, h), "down": (h, 21504), "lm_head": (262144, h)}
    out = []
    for name, (N, K) in shapes.items():
        if only and name not in only.split(","):
            continue
        w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
        lin = L.Linear(w, "bf16")
        for t in tokens:
            x = torch.randn(t, K, device=dev).to(torch.bfloat16)
            ours = _time_flushed(lambda: lin(x))
            cub = _time_flushed(lambda: Fn.linear(x, w))
            wbytes = N * K * 2
            nt = L.FORCE["nt"] or MG.pick_nt(t)
            ks = L.FORCE["ks"] or L.split_k(N // (128 * lin.lin.g), t, nt, K // 64, lin.lin.num_ctas, g=lin.lin.g)
            row = {"op": name, "N": N, "K": K, "tokens": t, "nt": nt, "ksplit": ks, "ours_us": round(ours, 1),
                   "cublas_us": round(cub, 1), "ours_frac_hbm": round(wbytes / ours / 1e3 / PEAKS["hbm_gbs"], 3),
                   "cublas_frac_hbm": round(wbytes / cub / 1e3 / PEAKS["hbm_gbs"], 3),
                   "kernels_us": _kernel_times(lambda: lin(x))}
            out.append(row)
        del lin, w
    return out


def _gemm_trace(fn) -> dict:
    """CTA 0's phase timeline (clock64 cycles from kernel start) of the LAST GEMM launch of one fn() call, L2 flushed
    before the call (`MgTraceEv` order in csrc/kernels.h)."""
    from ..ops import moe_gemm as MG
    names = ["start", "setup", "first_copy", "first_ready", "last_mma", "acc_seen", "epi_done", "end"] + [
        f"c{c}_{k}" for c in range(3) for k in ("tmem", "staged", "stored", "_")]
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    tr = torch.zeros(len(names), dtype=torch.int64, device="cuda")
    torch.sum(flush, dim=0, out=sink)
    MG.TRACE[0] = tr
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        MG.TRACE[0] = None
    v = tr.cpu().tolist()
    return {n: int(x - v[0]) for n, x in zip(names, v)}


def _kernel_times(fn, reps: int = 5) -> dict:
    """Mean device duration per kernel name of one fn() call (CUDA activity records of the torch profiler, L2
    flushed before each call): the kernel-only split of a call that also has CPU launch gaps."""
    from torch.profiler import ProfilerActivity, profile
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)
            fn()
        torch.cuda.synchronize()
    res = {}
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", None)
        if t is None:
            t = getattr(e, "cuda_time_total", 0)
        if t > 0 and "reduce_kernel<" not in e.key:
            k = e.key.split("(")[0].replace("void ", "").replace("iob::(anonymous namespace)::", "")[:48]
            res[k] = round(res.get(k, 0.0) + t / reps, 2)
    return res


def _graph_time_flushed(fn, iters: int = 20) -> float:
    """Mean device time of one CUDA-graph replay of fn (captured after two warm-up calls), L2 flushed by a 512 MB
    read before each replay (not timed)."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return _time_flushed(g.replay, iters)


def kv4mla_compare_case(tokens: list, topk: int = 2048, rows: int = 600000, heads: int = 64) -> list:
    """This framework's sparse-MLA decode (csrc/attn_mla_decode.cu) against the reference's own sm_100 kernel
    (kv4mla, fp8 mode), same box, same shapes: NVFP4 352-byte rows, `rows`-row pool, top-`topk` random rows per
    token, `heads` query heads; both fed the same E4M3 query values, each replayed from a CUDA graph with the L2
    flushed in between.  The reference module is the reference repository's kernel compiled unmodified into
    baseline/kv4mla_build/ (git-ignored); absent -> the row says so."""
    import glob
    import importlib.util
    from ..ops import kvcache as K
    from ..ops import mla as M
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    so = sorted(glob.glob(os.path.join(root, "baseline", "kv4mla_build", "*", "kv4mla_ext_*.so")))
    if not so:
        return [{"kernel": "kv4mla_compare", "unavailable": "reference module not built into baseline/kv4mla_build"}]
    spec = importlib.util.spec_from_file_location(os.path.basename(so[0]).split(".")[0], so[0])
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda:0")
    pool = mla_pool_random(rows, K.FMT_NVFP4, dev)
    parts = int(ref.num_sm_parts(1))
    sm = 1.0 / math.sqrt(576)
    out_rows = []
    for t in tokens:
        g = torch.Generator(device=dev).manual_seed(t)
        idx = torch.randint(0, rows, (t, topk), generator=g, device=dev, dtype=torch.int32)
        q8 = (torch.randn(t, heads, 576, generator=g, device=dev)).to(torch.float8_e4m3fn)
        qb = q8.float().to(torch.bfloat16)                       # the same query values for both kernels
        ours_out = torch.empty(t, heads, 512, dtype=torch.bfloat16, device=dev)
        splits = M.mla_split_policy(t, topk)
        ws = M.MlaWorkspace.allocate(t, heads, splits[0], device=dev)

        def ours():
            M.mla_decode(qb, pool, idx, sm, K.FMT_NVFP4, splits=splits, ws=ws, out=ours_out)
        # the reference's split rule (kv4mla.py split_policy / sched_overhead), its workspace layout
        split = topk > 640 and not (96 <= t <= 136 or t >= 224)
        ref_out = torch.empty(t, 1, heads, 512, dtype=torch.bfloat16, device=dev)
        ref_lse = torch.empty(t, 1, heads, dtype=torch.float32, device=dev)
        meta = ns = oa = la = None
        if split:
            meta = torch.empty(parts, 8, dtype=torch.int32, device=dev)
            ns = torch.empty(t + 1, dtype=torch.int32, device=dev)
            ref.sched_meta(t, 1, topk, None, meta, ns, 10 if t <= 16 else 5)
            oa = torch.empty(t + parts, 1, heads, 512, dtype=torch.float32, device=dev)
            la = torch.empty(t + parts, 1, heads, dtype=torch.float32, device=dev)
        q4 = q8.view(t, 1, heads, 576)
        idx3 = idx.view(t, 1, topk)

        def theirs():
            ref.sparse_decode(q4, pool, idx3, None, float(sm), ref_out, ref_lse, meta, ns, oa, la, True)
        us_ours = _graph_time_flushed(ours)
        us_ref = _graph_time_flushed(theirs)
        ours()
        theirs()
        torch.cuda.synchronize()
        cos = torch.nn.functional.cosine_similarity(ours_out.float().flatten(), ref_out.float().flatten(), dim=0)
        out_rows.append({"kernel": "kv4mla_compare", "tokens": t, "heads": heads, "topk": topk, "pool_rows": rows,
                         "ours_us": round(us_ours, 2), "kv4mla_us": round(us_ref, 2),
                         "ratio_ref_over_ours": round(us_ref / us_ours, 3), "ours_splits": list(splits),
                         "kv4mla_split": split, "output_cosine": round(cos.item(), 5)})
    return out_rows


def dsa_profile_case(layers: int, sessions: int, ctx: int, steps: int, prefill: int, top: int = 40,
                     trace_out: str = "", model: str = "dsa_moe") -> dict:
    """Per-kernel device time of the DSA-MoE serving step (the bench's engine: DP attention + EP over the launched
    ranks, CUDA-graph decode), from the CUDA activity records of the torch profiler (kernel durations as CUPTI reports
    them; the shares, not the absolutes, are the point: the bench's own CUDA-event timing is the throughput figure).
    Sessions hold `ctx` positions of random well-formed KV written by the pool writers (no prefill compute before the
    decode steps); with `prefill` > 0 one more request of that many tokens per rank is prefilled and profiled too.
    `trace_out`: also write rank 0's decode-step activity as a Chrome trace (kernel order, starts and gaps).
    `model`: the MLA + DSA + MoE preset (`dsa_moe`, or `glm5` for the long-context geometry)."""
    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile
    from ..config import EngineConfig, model_config
    from ..engine.engine import Engine
    from ..engine.scheduler import SamplingParams
    from ..engine.synthetic import synth_mla_sessions
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    per = sessions // world
    cfg = model_config(model, num_layers=layers)
    ecfg = EngineConfig(model=model, device=str(dev), kv_dtype="nvfp4", max_running=per + 1,
                        chunked_prefill=max(prefill, 64), graph_batch_sizes=str(per), ep=world, prefix_cache=False)
    eng = Engine(ecfg, cfg, max_seq=ctx + max(prefill, 0) + 256, ep_rank=rank,
                 ep_group=dist.group.WORLD if world > 1 else None)
    synth_mla_sessions(eng, per, ctx, 200, seed=1 + rank)
    eng.runner.warm_graphs(per)
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()

    def table(prof, n):
        rows = []
        for e in prof.key_averages():
            t = getattr(e, "device_time_total", None)
            if t is None:
                t = getattr(e, "cuda_time_total", 0)
            if t > 0 and e.count > 0:
                rows.append((e.key[:110], t / n, e.count // n))
        rows.sort(key=lambda r: -r[1])
        tot = sum(r[1] for r in rows)
        return {"total_us": round(tot, 1), "kernels": [{"name": k, "us": round(u, 1), "launches": c,
                                                          "share": round(u / tot, 4)} for k, u, c in rows[:top]]}
    res = {"layers": layers, "sessions": sessions, "ctx": ctx, "world": world}
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            eng.step()
        torch.cuda.synchronize()
    res["decode_step"] = table(prof, steps)
    if trace_out and rank == 0:
        prof.export_chrome_trace(trace_out)
    if prefill:
        g = torch.Generator().manual_seed(7 + rank)
        eng.add_request(torch.randint(1, cfg.vocab, (prefill,), generator=g).tolist(), SamplingParams(max_new_tokens=4))
        eng.sched.burst = 1
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            eng.step()
            torch.cuda.synchronize()
        res["prefill_chunk"] = table(prof, 1)
        res["prefill_chunk"]["tokens"] = prefill
    return res if rank == 0 else {}


def main() -> None:
    _load_peaks()
    p = argparse.ArgumentParser()
    p.add_argument("kernel")
    p.add_argument("--b", type=int, default=8)
    p.add_argument("--hk", type=int, default=16)
    p.add_argument("--hq", type=int, default=32)
    p.add_argument("--heads", type=int, default=128)
    p.add_argument("--d", type=int, default=512)
    p.add_argument("--ctx", type=int, default=8192)
    p.add_argument("--fmt", default="nvfp4")
    p.add_argument("--nq", type=int, default=1)
    p.add_argument("--chunk", type=int, default=2048)
    p.add_argument("--splits", default="", help="gqa_decode: force (num_splits,tiles_per_split); mla_decode: "
                                                "';'-separated list of such pairs to sweep")
    p.add_argument("--window", type=int, default=0)
    p.add_argument("--topk", type=int, default=2048)
    p.add_argument("--launches", type=int, default=0)
    p.add_argument("--trace", action="store_true", help="gqa_decode: per-tile clock64 timeline of CTA 0")
    p.add_argument("--experts", type=int, default=32)
    p.add_argument("--total-experts", type=int, default=256)
    p.add_argument("--hidden", type=int, default=7168)
    p.add_argument("--ffn", type=int, default=2048)
    p.add_argument("--wfmt", default="fp8", choices=["fp8", "nvfp4"])
    p.add_argument("--layers", type=int, default=13)
    p.add_argument("--sessions", type=int, default=64)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--prefill", type=int, default=0)
    p.add_argument("--tokens", default="8,64,8192")
    p.add_argument("--only", default="", help="proj_gemms: comma-separated op names")
    p.add_argument("--nt", default="", help="proj_gemms: token tiles to sweep (comma-separated)")
    p.add_argument("--ks", default="", help="proj_gemms: K splits to sweep (comma-separated)")
    p.add_argument("--trace-out", default="", help="dsa_profile: Chrome trace of the decode steps (rank 0)")
    p.add_argument("--model", default="dsa_moe", help="dsa_profile: MLA + DSA + MoE preset")
    a = p.parse_args()
    if a.kernel == "gqa_decode":
        r = gqa_decode_case(a.b, a.hk, a.hq, a.d, a.ctx, a.fmt, a.nq, a.window, a.launches, a.splits, a.trace)
    elif a.kernel == "gqa_extend":
        r = gqa_extend_case(a.chunk, a.ctx, a.hk, a.hq, a.d, a.fmt, a.window, a.launches)
    elif a.kernel == "indexer":
        r = indexer_case(a.b, a.ctx, a.topk, launches=a.launches)
    elif a.kernel == "hotops":
        r = {}
        for op in a.only.split(",") if a.only else ("rmsnorm_fp8", "router", "kv_write"):
            for t in [int(v) for v in a.tokens.split(",")]:
                row = hotops_case(op, t, launches=a.launches)
                if row:
                    print(json.dumps(row), flush=True)
    elif a.kernel == "moe_tactics":
        r = moe_tactics_case(a.experts, a.total_experts, a.topk, a.hidden, a.ffn, a.wfmt)
    elif a.kernel == "dense_linear":
        r = dense_linear_case(a.b, a.launches)
    elif a.kernel == "ep_moe":
        import torch.distributed as dist
        rank = int(os.environ.get("RANK", "0"))
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
        r = ep_moe_case(a.b, a.total_experts, a.topk, a.hidden, a.ffn, a.wfmt)
        dist.barrier()
        dist.destroy_process_group()
        if rank:
            r = {}
    elif a.kernel == "tp_gemm_ar":
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
        for row in tp_gemm_ar_case([int(v) for v in a.tokens.split(",")], a.ffn, a.hidden):
            print(json.dumps(row), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        r = {}
    elif a.kernel == "moe_gemm":
        r = moe_gemm_case(a.b, a.experts, a.total_experts, a.topk, a.hidden, a.ffn, a.wfmt, a.launches)
    elif a.kernel == "proj_gemms":
        from ..ops import linear as L
        for nt in [int(v) for v in a.nt.split(",")] if a.nt else [None]:
            for ks in [int(v) for v in a.ks.split(",")] if a.ks else [None]:
                L.FORCE.update(nt=nt, ks=ks)
                for row in proj_gemms_case([int(v) for v in a.tokens.split(",")], a.only):
                    row.update(nt=nt, ks=ks)
                    print(json.dumps(row), flush=True)
        L.FORCE.update(nt=None, ks=None)
        r = {}
    elif a.kernel == "dense_gemms":
        from ..ops import linear as L
        for nt in [int(v) for v in a.nt.split(",")] if a.nt else [None]:
            for ks in [int(v) for v in a.ks.split(",")] if a.ks else [None]:
                L.FORCE.update(nt=nt, ks=ks)
                for row in dense_gemms_case([int(v) for v in a.tokens.split(",")], a.only):
                    print(json.dumps(row), flush=True)
        L.FORCE.update(nt=None, ks=None)
        r = {}
    elif a.kernel == "kv4mla_compare":
        for row in kv4mla_compare_case([int(v) for v in a.tokens.split(",")], a.topk, heads=a.heads):
            print(json.dumps(row), flush=True)
        r = {}
    elif a.kernel == "dsa_profile":
        import torch.distributed as dist
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world > 1:
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
            dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
        r = dsa_profile_case(a.layers, a.sessions, a.ctx, a.steps, a.prefill, trace_out=a.trace_out, model=a.model)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    elif a.kernel == "mla_decode":
        for sp in (a.splits.split(";") if a.splits else [""]):
            row = mla_decode_case(a.b, a.heads, a.ctx, a.topk, a.fmt, a.nq, a.launches, sp)
            if row:
                print(json.dumps(row), flush=True)
        r = {}
    else:
        raise SystemExit(f"unknown kernel {a.kernel}")
    if r:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
