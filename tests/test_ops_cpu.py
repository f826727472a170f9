"""CPU oracle consistency: pool write/read round trip, paged decode oracle vs dense attention, op references."""
import math

import torch

from inference_optimizations_b200.ops import attention as A
from inference_optimizations_b200.ops import basic as B
from inference_optimizations_b200.ops import kvcache as K


def test_swizzle_perm_is_permutation():
    for rb in (64, 128, 256, 512, 1024):
        p = K.kv_swizzle_perm(rb)
        for r in range(64):
            assert sorted(p[r].tolist()) == list(range(rb))


def test_pool_roundtrip_all_formats():
    torch.manual_seed(0)
    hk, d, n = 2, 256, 150
    for fmt in (K.FMT_BF16, K.FMT_FP8, K.FMT_NVFP4):
        pool = torch.zeros(4, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8)
        pages = torch.tensor([2, 0, 3])
        k = torch.randn(n, hk, d).to(torch.bfloat16).float()
        v = torch.randn(n, hk, d).to(torch.bfloat16).float()
        pos = torch.arange(n)
        K.gqa_pool_write_ref(pool, pages[pos // 64] * 64 + pos % 64, k, v, fmt, 0.5, 0.5)
        k2, v2 = K.gqa_pool_read_ref(pool, pages, n, fmt, d, 0.5, 0.5)
        tol = {K.FMT_BF16: 0.0, K.FMT_FP8: 0.3, K.FMT_NVFP4: 0.7}[fmt]
        assert (k2 - k).abs().max() <= tol + 1e-6 and (v2 - v).abs().max() <= tol + 1e-6


def test_decode_ref_matches_dense():
    torch.manual_seed(1)
    hq, hk, d, n_q = 4, 2, 128, 3
    lens = [70, 5]
    fmt = K.FMT_BF16
    pool = torch.zeros(6, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8)
    pt = torch.tensor([[1, 4], [0, 5]], dtype=torch.int32)
    ks, vs = [], []
    for i, n in enumerate(lens):
        k = torch.randn(n, hk, d).to(torch.bfloat16).float()
        v = torch.randn(n, hk, d).to(torch.bfloat16).float()
        pos = torch.arange(n)
        K.gqa_pool_write_ref(pool, pt[i][pos // 64].long() * 64 + pos % 64, k, v, fmt)
        ks.append(k)
        vs.append(v)
    q = torch.randn(len(lens) * n_q, hq, d).to(torch.bfloat16)
    sm = 1 / math.sqrt(d)
    for window in (0, 4):
        out = A.gqa_decode_ref(q, pool, pt, torch.tensor(lens), n_q, hk, fmt, sm, window)
        for i, n in enumerate(lens):
            qp = torch.arange(n - n_q, n)
            ref = A.dense_attention_ref(q[i * n_q:(i + 1) * n_q], ks[i], vs[i], sm, qp, torch.arange(n), window)
            assert torch.allclose(out[i * n_q:(i + 1) * n_q], ref, atol=1e-5)


def test_split_policy():
    ns, tps = A.split_policy(32 * 16, 33000)
    assert ns * tps * 128 >= 33000 and ns >= 1
    ns, tps = A.split_policy(4, 200000)
    assert ns > 1 and tps >= 4
    ns, tps = A.split_policy(512, 1030, window=1024)
    assert ns * tps * 128 >= 1024 + 128


def test_rmsnorm_and_argmax_ref():
    x = torch.randn(3, 64).to(torch.bfloat16)
    w = torch.zeros(64).to(torch.bfloat16)
    y = B.rmsnorm(x, w, 1e-6, plus_one=True)
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(y.float(), ref, atol=2e-2)
    lg = torch.tensor([[1.0, 3.0, 3.0, 0.0]])
    assert B.argmax(lg).tolist() == [1]


def test_index_pool_layout_roundtrip():
    from inference_optimizations_b200.ops import formats as F
    from inference_optimizations_b200.ops import kvcache as K
    torch.manual_seed(0)
    k = torch.randn(150, 128).to(torch.bfloat16)
    slot = torch.randperm(3 * 64)[:150].int()
    slot[7] = -1
    pool = torch.zeros(3, K.INDEX_PAGE_BYTES, dtype=torch.uint8)
    K.index_key_write(k, slot, pool)
    keep = slot >= 0
    assert torch.equal(K.index_key_read(pool, slot[keep]), F.index_key_quantize(k[keep].float()))
    # values of one page form a 128-byte-swizzled [64 x 128] tile: chunk c of row r at c ^ (r & 7)
    r, c = 13, 3
    page = pool[0]
    rows = F.index_key_quantize(k.float())
    pos = (slot == r).nonzero()
    if len(pos):
        i = int(pos[0])
        assert torch.equal(page[r * 128 + ((c ^ (r & 7)) * 16): r * 128 + ((c ^ (r & 7)) * 16) + 16], rows[i, 16 * c:16 * c + 16])


def test_ep_layout_regions_and_pair_routing():
    from inference_optimizations_b200.parallel.ep import EPLayout
    for fmt in ("fp8", "nvfp4"):
        L = EPLayout(world=8, T_max=16, topk=8, H=7168, fmt=fmt)
        regions = [(L.off_x, 8 * 16 * L.row_bytes), (L.off_s, 8 * 16 * L.scale_words * 4),
                   (L.off_ids, 8 * 16 * 8 * 4), (L.off_comb, L.comb_rows * 7168 * 2), (L.off_flags, 8 * 4)]
        for (a, n), (b, _) in zip(regions, regions[1:]):
            assert a % 256 == 0 and a + n <= b
        assert L.off_flags + 32 <= L.nbytes
        # every pair's output lands on the rank that owns its token, at row t * topk + k
        for src in (0, 3, 7):
            for t in (0, 5, 15):
                for k in (0, 7):
                    assert L.comb_row(L.pair(src, t, k)) == (src, t * 8 + k)
        assert L.owner(255, 32) == 7 and L.owner(32, 32) == 1


def test_act_quant_ref_roundtrip():
    """CPU path of the fused activation + quant: dequantized output tracks act_mul within the format's error."""
    import torch
    from inference_optimizations_b200.ops import basic as B
    from inference_optimizations_b200.ops import moe_gemm as MG
    from inference_optimizations_b200.ops.linear import act_quant
    torch.manual_seed(0)
    gu = torch.randn(5, 512).to(torch.bfloat16)
    a = B.act_mul(gu, True).float()
    q, s = act_quant(gu, True, 0)
    assert q.shape == (5, 256) and s.shape == (5, 2)
    d = MG.dequant_rows(q, s)
    assert ((d - a).abs() <= a.abs().amax(-1, keepdim=True) / 16 + 1e-6).all()
    q4, s4 = act_quant(gu, False, 1)
    assert q4.shape == (5, 128) and s4.shape == (5, 4)
    d4 = MG.dequant_nvfp4_rows(q4, s4)
    a4 = B.act_mul(gu, False).float()
    assert (d4 - a4).abs().max() <= a4.abs().max() / 3


def test_extend_blocks_and_oracle_match_decode_oracle():
    """The extend work list covers every prefill token once, and the extend oracle equals the decode oracle run
    token by token over the same pool."""
    import math
    import torch
    from inference_optimizations_b200.ops import attention as A
    from inference_optimizations_b200.ops import kvcache as K
    assert A.extend_blocks([(0, 150, 10, 3)], 2) == [(0, 64, 10, 3), (64, 64, 74, 3), (128, 22, 138, 3)]
    torch.manual_seed(0)
    d, hk, hq, n = 128, 1, 2, 90
    pool = torch.zeros(4, hk, 2, K.part_bytes(K.FMT_FP8, d), dtype=torch.uint8)
    pt = torch.tensor([[2, 0]], dtype=torch.int32)
    k = torch.randn(n, hk, d).to(torch.bfloat16).float()
    v = torch.randn(n, hk, d).to(torch.bfloat16).float()
    pos = torch.arange(n)
    K.gqa_pool_write_ref(pool, pt[0][pos // 64].long() * 64 + pos % 64, k, v, K.FMT_FP8)
    q = torch.randn(30, hq, d).to(torch.bfloat16)
    blocks = torch.tensor(A.extend_blocks([(0, 30, 60, 0)], hq // hk), dtype=torch.int32)
    for w in (0, 17):
        ext = A.gqa_extend_ref(q, pool, pt, blocks, hk, K.FMT_FP8, 1 / math.sqrt(d), w)
        dec = A.gqa_decode_ref(q, pool, pt.repeat(30, 1), torch.arange(61, 91, dtype=torch.int32), 1, hk, K.FMT_FP8,
                               1 / math.sqrt(d), w)
        assert torch.allclose(ext, dec, atol=1e-5)
