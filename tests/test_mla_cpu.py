"""Sparse MLA (DSA) decode on CPU: the fp32 oracle and the CPU plumbing config (NVFP4 KV quantize + dequant-gather +
sparse MLA decode against unquantized attention), plus the split planner."""
import math

import torch

from inference_optimizations_b200.ops import formats as F
from inference_optimizations_b200.ops import mla as M
from inference_optimizations_b200.ops.kvcache import FMT_FP8, FMT_NVFP4


def test_config1_nvfp4_sparse_decode_vs_unquantized():
    torch.manual_seed(0)
    b, h, n, topk = 4, 16, 4096, 2048
    nope = torch.randn(b * n, 512)
    rope = torch.randn(b * n, 64)
    pool = F.mla_row_quantize(nope, rope)                           # [b*n, 352]
    assert pool.shape == (b * n, 352)
    scores = torch.randn(b, n)                                      # random-normal indexer
    pos = scores.topk(topk, dim=-1).indices
    idx = (pos + torch.arange(b)[:, None] * n).int()
    q = torch.randn(b, h, 576)
    sm = 1.0 / math.sqrt(576)
    out, lse = M.mla_decode(q, pool, idx, sm, FMT_NVFP4, return_lse=True)
    kv = torch.cat([nope, rope], dim=-1)
    exact, exact_lse = F.sparse_mla_reference(q, kv, idx, sm)
    # 4-bit latents: per-element relative error <= 1/4 of the block's step; the attention output is an average of
    # ~2048 rows, so its error shrinks well below that
    rel = (out.float() - exact).norm() / exact.norm()
    assert rel < 0.12, rel
    assert (lse - exact_lse).abs().max() < 0.1
    # FP8 rows on the same indices are closer still
    pool8 = F.mla_fp8_row_quantize(nope, rope)
    out8 = M.mla_decode(q, pool8, idx, sm, FMT_FP8)
    rel8 = (out8.float() - exact).norm() / exact.norm()
    assert rel8 < rel and rel8 < 0.05, rel8


def test_reference_masks_and_matches_dense():
    torch.manual_seed(1)
    rows, t, h, topk = 300, 3, 4, 40
    pool = F.mla_row_quantize(torch.randn(rows, 512), torch.randn(rows, 64))
    idx = torch.stack([torch.randperm(rows)[:topk] for _ in range(t)]).int()
    idx[0, ::3] = -1
    idx[2] = -1
    q = torch.randn(t, h, 576)
    out, lse = M.mla_decode_ref(q, pool, idx, 0.1)
    kv = F.mla_row_dequantize(pool)
    for i in range(2):
        sel = idx[i][idx[i] >= 0].long()
        s = q[i] @ kv[sel].T * 0.1
        assert torch.allclose(out[i], torch.softmax(s, -1) @ kv[sel, :512], atol=1e-5)
        assert torch.allclose(lse[i], torch.logsumexp(s, -1), atol=1e-5)
    assert out[2].abs().max() == 0 and torch.isinf(lse[2]).all()


def test_split_policy_fills_sms():
    assert M.mla_split_policy(64, 2048) == (1, 2048 // M.TILE)     # 128 CTAs: one wave already
    ns, tps = M.mla_split_policy(1, 2048)
    assert ns * tps * M.TILE >= 2048 and 2 * ns <= 148 and ns > 4
    ns, tps = M.mla_split_policy(8, 200)
    assert ns * tps * M.TILE >= 200


def test_dense_mla_indices_and_decode():
    """Dense mode: indices from the page table cover exactly [0, kv_len); decode equals sparse decode over them."""
    import math
    from inference_optimizations_b200.ops import formats as F
    from inference_optimizations_b200.ops import mla as M
    torch.manual_seed(2)
    pages = torch.randperm(20)[:12].view(3, 4).int()
    kv_len = torch.tensor([70, 256, 1], dtype=torch.int32)
    idx = M.dense_indices(pages, kv_len, 256)
    assert idx.shape == (3, 256)
    for b in range(3):
        n = int(kv_len[b])
        want = (pages[b].long()[torch.arange(n) // 64] * 64 + torch.arange(n) % 64).int()
        assert torch.equal(idx[b, :n], want) and torch.all(idx[b, n:] == -1)
    pool = F.mla_row_quantize(torch.randn(20 * 64, 512), torch.randn(20 * 64, 64))
    q = torch.randn(3, 4, 576).to(torch.bfloat16)
    sm = 1 / math.sqrt(576)
    o1 = M.mla_dense_decode(q, pool, pages, kv_len, sm)
    o2, _ = M.mla_decode_ref(q, pool, idx, sm, M.FMT_NVFP4)
    assert torch.allclose(o1.float(), o2.float(), atol=1e-2)


def test_mla_latent_and_expanded_layouts_agree():
    """Absorbed latent (MQA over 576-dim rows) and expanded per-head MHA (padded to 256) give the same attention to
    1e-9 in fp64, with a causal mask."""
    import torch
    from inference_optimizations_b200.ops import mla as M
    torch.manual_seed(0)
    t, s, h, dn, dr, dv, lat = 5, 40, 4, 128, 64, 128, 512
    d = torch.float64
    q_nope, q_pe = torch.randn(t, h, dn, dtype=d), torch.randn(t, h, dr, dtype=d)
    c_kv, k_pe = torch.randn(s, lat, dtype=d), torch.randn(s, dr, dtype=d)
    w_uk, w_uv = torch.randn(h, dn, lat, dtype=d) * 0.05, torch.randn(h, lat, dv, dtype=d) * 0.05
    mask = torch.arange(s)[None, :] <= (torch.arange(t)[:, None] + s - t)
    a = M.mla_attention_latent(q_nope, q_pe, c_kv, k_pe, w_uk, w_uv, 192 ** -0.5, mask)
    b = M.mla_attention_expanded(q_nope, q_pe, c_kv, k_pe, w_uk, w_uv, 192 ** -0.5, mask)
    assert a.shape == (t, h, dv) and (a - b).abs().max().item() < 1e-9
    k, v = M.mla_expand_kv(c_kv, k_pe, w_uk, w_uv)
    assert k.shape == (s, h, 256) and torch.all(k[..., dn + dr:] == 0) and torch.all(v[..., dv:] == 0)


def test_bf16_reference_pool_attention_matches_oracle():
    """Unquantized bf16 latent rows (the accuracy reference pool): the chunked fp32 attention equals the per-token
    oracle over the same rows, masked slots and a token with no valid row included, on any device."""
    from inference_optimizations_b200.ops import formats as F
    from inference_optimizations_b200.ops import kvcache as K
    from inference_optimizations_b200.ops import mla as M
    torch.manual_seed(7)
    rows, t, h, topk = 300, 5, 4, 40
    pool = torch.zeros(rows, F.MLA_BF16_ROW_BYTES, dtype=torch.uint8)
    nope, rope = torch.randn(rows, 512), torch.randn(rows, 64)
    K.mla_write(nope, rope, torch.arange(rows), pool)
    back = M.dequant_rows(pool, M.FMT_BF16)
    assert torch.equal(back, torch.cat([nope, rope], -1).to(torch.bfloat16).float())
    q = torch.randn(t, h, 576).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(rows)[:topk] for _ in range(t)]).int()
    idx[torch.rand(t, topk) < 0.2] = -1
    idx[3] = -1
    sm = M.mla_sm_scale()
    o, lse = M.mla_decode_exact(q, pool, idx, sm, chunk=2)
    ro, rl = F.sparse_mla_reference(q.float(), back, idx, sm)
    assert torch.allclose(o, ro, atol=1e-5, rtol=1e-5) and torch.equal(o[3], torch.zeros_like(o[3]))
    assert torch.allclose(lse, rl, atol=1e-5) and torch.isinf(lse[3]).all()
    out = M.mla_decode(q, pool, idx, sm, M.FMT_BF16)
    assert torch.allclose(out.float(), ro.to(torch.bfloat16).float(), atol=2e-2)


def test_mla_engine_latent_pool_formats():
    """kv_dtype picks the latent row: nvfp4 352 B, fp8 576 B, bf16 1152 B (unquantized, the reference: torch
    attention path, no graphs); the three engines share weights and agree closely on prefill logits; an unknown
    kv_dtype is refused."""
    import pytest
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import Request, SamplingParams, Segment
    cfg = model_config("tiny_mla")
    engines = {}
    for kv in ("bf16", "fp8", "nvfp4"):
        ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype=kv, max_running=2, chunked_prefill=64)
        engines[kv] = Engine(ecfg, cfg, max_seq=128)
    assert [engines[k].runner.kv.latent[0].shape[1] for k in ("bf16", "fp8", "nvfp4")] == [1152, 576, 352]
    assert engines["bf16"].runner.ref_pool and not engines["bf16"].runner._graphable()
    torch.manual_seed(1)
    prompt = torch.randint(1, cfg.vocab, (60,)).tolist()
    logits = {}
    for kv, eng in engines.items():
        if kv != "bf16":
            eng.runner.model.copy_from(engines["bf16"].runner.model)
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        logits[kv] = eng.runner.model.logits(eng.runner.model.forward(st, eng.runner.kv)).float()
        eng.runner.detach(r)
    for kv in ("fp8", "nvfp4"):
        cos = torch.nn.functional.cosine_similarity(logits[kv], logits["bf16"], dim=-1)
        assert cos.min().item() > 0.9, (kv, cos.min().item())
    out = engines["bf16"].generate([prompt[:30]], SamplingParams(max_new_tokens=4))
    assert len(out[0]) == 4
    with pytest.raises(ValueError):
        Engine(EngineConfig(model="tiny_mla", device="cpu", kv_dtype="int4", max_running=2), cfg, max_seq=128)


def test_exact_attention_over_quantized_rows_matches_oracle():
    """The exact-arithmetic arm: fp32 attention over NVFP4 / FP8 rows decoded exactly equals the per-token oracle
    over the same dequantized rows."""
    from inference_optimizations_b200.ops import formats as F
    from inference_optimizations_b200.ops import kvcache as K
    from inference_optimizations_b200.ops import mla as M
    torch.manual_seed(9)
    rows, t, h, topk = 200, 4, 4, 32
    nope, rope = torch.randn(rows, 512), torch.randn(rows, 64)
    q = torch.randn(t, h, 576).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(rows)[:topk] for _ in range(t)]).int()
    idx[torch.rand(t, topk) < 0.25] = -1
    sm = M.mla_sm_scale()
    for fmt, width in ((M.FMT_NVFP4, F.MLA_ROW_BYTES), (M.FMT_FP8, F.MLA_FP8_ROW_BYTES)):
        pool = torch.zeros(rows, width, dtype=torch.uint8)
        K.mla_write(nope, rope, torch.arange(rows), pool)
        o, lse = M.mla_decode_exact(q, pool, idx, sm, fmt, chunk=3)
        ro, rl = M.mla_decode_ref(q, pool, idx, sm, fmt)
        assert torch.allclose(o, ro, atol=1e-5, rtol=1e-5) and torch.allclose(lse, rl, atol=1e-5)
