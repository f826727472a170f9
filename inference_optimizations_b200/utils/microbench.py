"""Kernel microbenchmarks (CUDA-event timed, warm, inputs larger than L2 unless stated) for the ncu summaries in
profiles/.  Usage:

    python -m inference_optimizations_b200.utils.microbench gqa_decode --b 8 --ctx 8192 --d 512 --fmt nvfp4
    python -m inference_optimizations_b200.utils.microbench mla_decode --b 64 --heads 128 --ctx 131072 --fmt nvfp4

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
                    launches: int = 0) -> dict:
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
    ws = A.DecodeWorkspace.allocate(b, hk, splits[0], d, device=dev)

    def fn():
        A.gqa_decode(q, pool, pt, kv_len, n_q, hk, fmt, 1 / math.sqrt(d), window, splits=splits, ws=ws)
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
    p.add_argument("--window", type=int, default=0)
    p.add_argument("--topk", type=int, default=2048)
    p.add_argument("--launches", type=int, default=0)
    a = p.parse_args()
    if a.kernel == "gqa_decode":
        r = gqa_decode_case(a.b, a.hk, a.hq, a.d, a.ctx, a.fmt, a.nq, a.window, a.launches)
    elif a.kernel == "mla_decode":
        from ..ops.mla import mla_decode_case
        r = mla_decode_case(a.b, a.heads, a.ctx, a.topk, a.fmt, a.nq, a.launches, PEAKS)
    else:
        raise SystemExit(f"unknown kernel {a.kernel}")
    if r:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
