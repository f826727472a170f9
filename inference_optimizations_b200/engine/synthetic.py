"""Synthetic serving state for benchmarks: sessions that already hold a long prompt in the KV pool.

The pools are filled with random but well-formed rows (NVFP4 codes + E4M3 block scales in a realistic range, FP8
without NaN encodings, bf16 normals), so a decode step reads exactly the bytes and does exactly the math it would
after a real prefill; only the prompt's prefill compute is skipped (it is not part of a decode step).
"""
from __future__ import annotations

import torch

from ..ops import kvcache as K
from .scheduler import SamplingParams


def fill_pool_random(pool: torch.Tensor, fmt: int, d: int, seed: int) -> None:
    g = torch.Generator(device=pool.device)
    g.manual_seed(seed)
    flat = pool.view(-1, pool.shape[-1])
    step = max(1, (1 << 28) // pool.shape[-1])
    for i in range(0, flat.shape[0], step):
        blk = flat[i:i + step]
        if fmt == K.FMT_BF16:
            v = torch.randn(blk.shape[0], blk.shape[1] // 2, generator=g, device=pool.device).to(torch.bfloat16)
            blk.copy_(v.view(torch.uint8))
            continue
        blk.random_(0, 256, generator=g)
        if fmt == K.FMT_FP8:
            blk.bitwise_and_(0xBF)                       # exponent <= 7: |x| < 2, never the NaN code
        else:
            sc = blk[:, 64 * d // 2:]                    # E4M3 block scales: 0x20..0x2F = 0.125 .. 0.234
            sc.bitwise_and_(0x0F).bitwise_or_(0x20)


def synth_decode_sessions(engine, n: int, ctx: int, max_new: int, seed: int = 0) -> list:
    """Register n running requests whose first `ctx` tokens are in the pool and whose next input token is set."""
    runner, sched = engine.runner, engine.sched
    g = torch.Generator()
    g.manual_seed(seed)
    vocab = engine.cfg.vocab
    reqs = []
    for _ in range(n):
        prompt = torch.randint(1, vocab, (ctx,), generator=g).tolist()
        r = sched.new_request(prompt, SamplingParams(max_new_tokens=max_new))
        sched.waiting.remove(r)
        r.slot = sched.free_slots.pop()
        runner.attach(r)
        pg = runner.pages[r.rid]
        for k, rp in pg.items():
            if k.startswith("_"):
                continue
            if rp.window > 0:        # sliding-window kinds only ever hold the live window
                rp.high = max(0, (ctx - rp.window) // rp.page)
            rp.ensure(ctx)
            rp.trim(ctx)
        r.prefilled = r.kv_len = ctx
        r.pending = int(torch.randint(1, vocab, (1,), generator=g))
        r.output.append(r.pending)
        sched.running.append(r)
        reqs.append(r)
    runner.kv.sync_tables()
    for i, (pool, kind) in enumerate(zip(runner.kv.pools, runner.kv.kinds)):
        d = engine.cfg.head_dim_global if kind == "global" else engine.cfg.head_dim
        fill_pool_random(pool, runner.kv.fmt, d, seed * 7919 + i)
    if hasattr(runner, "after_synthetic"):
        runner.after_synthetic(reqs)
    return reqs


def synth_mla_sessions(engine, n: int, ctx: int, max_new: int, seed: int = 0, chunk: int = 1 << 16) -> list:
    """MLA family: register n running requests whose first `ctx` positions are in the latent and index pools (random
    latents / rope / index keys written through the pool writers, so every row is well formed) and whose next input
    token is set."""
    from ..ops import kvcache as K
    runner, sched = engine.runner, engine.sched
    cfg = engine.cfg
    g = torch.Generator()
    g.manual_seed(seed)
    reqs, slots = [], []
    for _ in range(n):
        prompt = torch.randint(1, cfg.vocab, (ctx,), generator=g).tolist()
        r = sched.new_request(prompt, SamplingParams(max_new_tokens=max_new))
        sched.waiting.remove(r)
        r.slot = sched.free_slots.pop()
        runner.attach(r)
        rp = runner.pages[r.rid]
        rp.ensure(ctx)
        slots += [rp.slot_of(p) for p in range(ctx)]
        r.prefilled = r.kv_len = ctx
        r.pending = int(torch.randint(1, cfg.vocab, (1,), generator=g))
        r.output.append(r.pending)
        sched.running.append(r)
        reqs.append(r)
    runner.kv.table.sync()
    dev = runner.device
    slot_t = torch.tensor(slots, dtype=torch.int32, device=dev)
    gd = torch.Generator(device=dev)
    gd.manual_seed(seed)
    for layer in range(len(runner.kv.latent)):
        for lo in range(0, slot_t.numel(), chunk):
            s = slot_t[lo:lo + chunk]
            m = s.numel()
            lat = torch.randn(m, cfg.kv_lora, generator=gd, device=dev).to(torch.bfloat16)
            rope = torch.randn(m, cfg.qk_rope, generator=gd, device=dev).to(torch.bfloat16)
            if getattr(runner.kv, "mixed", False):           # kvmix: slots past the split are NVFP4 rows
                sp = runner.kv.split_slot
                K.mla_write(lat, rope, torch.where(s < sp, s, torch.full_like(s, -1)), runner.kv.latent[layer])
                K.mla_write(lat, rope, torch.where(s >= sp, s - sp, torch.full_like(s, -1)), runner.kv.latent4[layer])
            else:
                K.mla_write(lat, rope, s, runner.kv.latent[layer])
            ik = torch.randn(m, cfg.index_dim, generator=gd, device=dev).to(torch.bfloat16)
            K.index_key_write(ik, s, runner.kv.index[layer])
    return reqs
