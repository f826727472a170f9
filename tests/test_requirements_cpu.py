"""Requirements that encode the reference's upstream correctness fixes (each one a behaviour this framework must
keep; `upstream-fixes/README.md:5-49` lists them):
  A1  a quantized KV scale is applied exactly once on the read path
  A2  an unquantized (bf16) cache ignores KV scales
  A3  the model's own routing function runs (softmax top-k renormalised)
  A5  decode and multi-token (extend / verify) attention use the same sliding-window rule
  A10 row offsets are 64-bit (pools beyond 2^31 bytes)
  humming-chunk: weight preparation quantizes one expert at a time
"""
import math

import torch

from inference_optimizations_b200.ops import attention as A
from inference_optimizations_b200.ops import kvcache as K
from inference_optimizations_b200.ops import moe as MOE


def _pool(fmt, d, lens, scale, seed=0):
    g = torch.Generator().manual_seed(seed)
    hk = 2
    per = max((n + 63) // 64 for n in lens)
    pt = torch.arange(1, 1 + len(lens) * per).view(len(lens), per).int()
    pool = torch.zeros(1 + len(lens) * per, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8)
    kv = []
    for i, n in enumerate(lens):
        k = torch.randn(n, hk, d, generator=g).to(torch.bfloat16).float()
        v = torch.randn(n, hk, d, generator=g).to(torch.bfloat16).float()
        slot = pt[i][torch.arange(n) // 64].long() * 64 + torch.arange(n) % 64
        K.gqa_pool_write_ref(pool, slot, k, v, fmt, scale, scale)
        kv.append((k, v))
    return pool, pt, torch.tensor(lens, dtype=torch.int32), kv


def test_a1_scale_applied_once():
    pool, pt, lens, kv = _pool(K.FMT_FP8, 128, [70], 4.0)
    k, v = K.gqa_pool_read_ref(pool, pt[0], 70, K.FMT_FP8, 128, 4.0, 4.0)
    assert ((k - kv[0][0]).abs().max() / kv[0][0].abs().max()) < 0.07      # not 4x (twice) or 1/4x (never)


def test_a2_bf16_cache_ignores_scales():
    pool, pt, lens, _ = _pool(K.FMT_BF16, 128, [50, 9], 1.0)
    q = torch.randn(2, 4, 128).to(torch.bfloat16)
    o1 = A.gqa_decode_ref(q, pool, pt, lens, 1, 2, K.FMT_BF16, 0.1, 0, 1.0, 1.0)
    o2 = A.gqa_decode_ref(q, pool, pt, lens, 1, 2, K.FMT_BF16, 0.1, 0, 3.0, 0.5)
    assert torch.equal(o1, o2)


def test_a3_softmax_router_renormalises():
    logits = torch.randn(9, 16)
    ids, w = MOE.route_ref(logits, torch.zeros(16), 4, 1, 1, 1.0, "softmax")
    assert torch.allclose(w.sum(-1), torch.ones(9))
    top = torch.softmax(logits, -1).topk(4, dim=-1).indices
    assert torch.equal(ids.long().sort(-1).values, top.sort(-1).values)


def test_a5_window_rule_same_for_decode_and_extend():
    d, w = 128, 40
    pool, pt, lens, _ = _pool(K.FMT_BF16, d, [100], 1.0)
    q = torch.randn(4, 4, d).to(torch.bfloat16)
    sm = 1 / math.sqrt(d)
    ext = A.gqa_decode_ref(q, pool, pt, lens, 4, 2, K.FMT_BF16, sm, w)            # 4 query tokens at 96..99
    for t in range(4):
        dec = A.gqa_decode_ref(q[t:t + 1], pool, pt, torch.tensor([97 + t], dtype=torch.int32), 1, 2, K.FMT_BF16,
                               sm, w)
        assert torch.allclose(ext[t], dec[0], atol=1e-6)


def test_a10_64bit_row_offsets():
    # the slot arithmetic of every pool stays in 64-bit integers: a page id past 2^31 / page bytes
    page = (1 << 31) // K.part_bytes(K.FMT_NVFP4, 512) + 5
    slot = torch.tensor([page * 64 + 3], dtype=torch.int64)
    off = slot.long() * (64 * 9)          # bytes of a 576-B row pool
    assert off.dtype == torch.int64 and int(off) > (1 << 31)


def test_expert_quantization_one_expert_at_a_time():
    from inference_optimizations_b200.ops import moe_gemm as MG
    w = torch.randn(3, 256, 256)
    q1, e1 = MG._quant_blocks_per_expert(w)
    q2, e2 = MG.quant_blocks(w)
    assert torch.equal(q1, q2) and torch.equal(e1, e2)


def test_indexer_selection_in_row_blocks_is_exact(monkeypatch):
    """Indexer logits chunked by rows (the reference's logits-OOM fix): a step whose fp32 score rows exceed the
    budget selects in blocks of token rows, with the same slots and positions as one pass (page-table rows by
    request index or, without one, by token)."""
    from inference_optimizations_b200.ops import indexer as I
    from inference_optimizations_b200.ops import kvcache as K
    torch.manual_seed(13)
    lens = [300, 700, 64, 500, 1, 0, 450]
    t = len(lens)
    per = max(-(-n // 64) for n in lens)
    pages = t * per + 2
    pt = torch.randperm(pages)[: t * per].view(t, per).int()
    pool = torch.zeros(pages, K.INDEX_PAGE_BYTES, dtype=torch.uint8)
    for i, n in enumerate(lens):
        if n:
            pos = torch.arange(n)
            K.index_key_write(torch.randn(n, 128).to(torch.bfloat16), (pt[i][pos // 64] * 64 + pos % 64).int(), pool)
    q8, w = I.indexer_q_quant(torch.randn(t, 8, 128), torch.rand(t, 8))
    limit = torch.tensor(lens, dtype=torch.int32)
    rix = torch.tensor([6, 5, 4, 3, 2, 1, 0], dtype=torch.int32)
    whole = [I.indexer_select(q8, w, pool, pt, limit if r is None else limit[r.long()], 128, 768, req_idx=r,
                              with_pos=True) for r in (None, rix)]
    monkeypatch.setattr(I, "SCORE_BYTES_MAX", 3 * 4 * 768)        # blocks of 3 rows
    blocks = [I.indexer_select(q8, w, pool, pt, limit if r is None else limit[r.long()], 128, 768, req_idx=r,
                               with_pos=True) for r in (None, rix)]
    for (s0, p0), (s1, p1) in zip(whole, blocks):
        assert torch.equal(s0, s1) and torch.equal(p0, p1)
