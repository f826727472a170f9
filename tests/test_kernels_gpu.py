"""sm_100a kernels against the fp32 torch oracles (bit-exact for quantized writes, toleranced for math)."""
import math

import pytest
import torch

from inference_optimizations_b200.ops import attention as A
from inference_optimizations_b200.ops import basic as B
from inference_optimizations_b200.ops import formats as F
from inference_optimizations_b200.ops import kvcache as K

pytestmark = pytest.mark.gpu


def test_umma_primitives(cuda):
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(0)
    for (m, n, k) in [(128, 16, 64), (256, 64, 256), (128, 256, 512)]:
        a = torch.randn(m, k, device=cuda).to(torch.bfloat16)
        b = torch.randn(n, k, device=cuda).to(torch.bfloat16)
        ref = a.float() @ b.float().T
        for sw64 in (0, 1):
            c = torch.empty(m, n, device=cuda)
            ext().umma_gemm_test(a, b, c, sw64)
            torch.cuda.synchronize()
            assert torch.allclose(c, ref, rtol=1e-3, atol=1e-2), (m, n, k, sw64, (c - ref).abs().max().item())


def test_umma_f8_mn_major(cuda):
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(0)
    for (n, k) in [(128, 128), (256, 256)]:
        a = torch.randn(128, k, device=cuda).to(torch.float8_e4m3fn)
        b = torch.randn(k, n, device=cuda).to(torch.float8_e4m3fn)
        c = torch.empty(128, n, device=cuda)
        ext().umma_f8_mn_test(a.view(torch.uint8), b.view(torch.uint8), c)
        torch.cuda.synchronize()
        ref = a.float() @ b.float()
        assert torch.allclose(c, ref, rtol=1e-4, atol=1e-3), (n, k, (c - ref).abs().max().item())


def test_nvfp4_lut_decode_bitexact(cuda):
    """The table decode used by the MLA kernel equals per-value conversion for every scale and nibble pattern."""
    from inference_optimizations_b200._ext import ext
    g = torch.Generator().manual_seed(0)
    nib = torch.arange(16, dtype=torch.int64)
    words = [(a | (b << 4)) * 0x01010101 for a in range(16) for b in range(16)]          # every nibble pair
    words += [int(nib[i % 16]) << (4 * (i % 8)) for i in range(128)]                    # single nibbles
    rnd = torch.randint(0, 2 ** 32, (8192,), generator=g, dtype=torch.int64)
    w = torch.tensor(words, dtype=torch.int64)
    w = torch.cat([w, rnd]) & 0xFFFFFFFF
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32).to(cuda)
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    ext().nvfp4_lut_test(w, out)
    torch.cuda.synchronize()
    assert out.item() == 0


@pytest.mark.parametrize("hidden,residual", [(5376, True), (7168, False), (256, True)])
def test_rmsnorm(cuda, hidden, residual):
    torch.manual_seed(1)
    x = torch.randn(7, hidden, device=cuda).to(torch.bfloat16)
    w = (torch.randn(hidden, device=cuda) * 0.1).to(torch.bfloat16)
    r = torch.randn(7, hidden, device=cuda).to(torch.bfloat16) if residual else None
    r_ref = r.cpu().clone() if residual else None
    y = B.rmsnorm(x, w, 1e-6, True, r)
    y_ref = B.rmsnorm(x.cpu(), w.cpu(), 1e-6, True, r_ref)
    assert torch.allclose(y.cpu().float(), y_ref.float(), rtol=2e-2, atol=2e-2)
    if residual:
        assert torch.equal(r.cpu(), r_ref)


def test_act_embed_argmax(cuda):
    torch.manual_seed(2)
    gu = torch.randn(5, 2 * 1024, device=cuda).to(torch.bfloat16)
    for gelu in (True, False):
        assert torch.allclose(B.act_mul(gu, gelu).cpu().float(), B.act_mul(gu.cpu(), gelu).float(),
                              rtol=2e-2, atol=2e-2)
    table = torch.randn(100, 256, device=cuda).to(torch.bfloat16)
    ids = torch.tensor([3, 99, 0, 3], device=cuda, dtype=torch.int32)
    assert torch.allclose(B.embed(ids, table, 16.0).cpu().float(), B.embed(ids.cpu(), table.cpu(), 16.0).float())
    logits = torch.randn(6, 262144, device=cuda).to(torch.bfloat16)
    logits[2, 777] = 100.0
    logits[2, 5] = 100.0  # tie: smallest index wins
    idx = B.argmax(logits)
    assert idx.cpu().tolist() == B.argmax(logits.cpu()).tolist()
    assert idx[2].item() == 5


@pytest.mark.parametrize("fmt", [K.FMT_NVFP4, K.FMT_FP8, K.FMT_BF16])
@pytest.mark.parametrize("d", [256, 512])
def test_gqa_prep_bitexact(cuda, fmt, d):
    torch.manual_seed(3)
    hq, hk, t = 4, 2, 70
    qkv = (torch.randn(t, (hq + 2 * hk) * d, device=cuda) * 2).to(torch.bfloat16)
    qn = (torch.randn(d, device=cuda) * 0.1).to(torch.bfloat16)
    kn = (torch.randn(d, device=cuda) * 0.1).to(torch.bfloat16)
    cs = B.rope_table(4096, d, 10000.0, cuda)
    pos = torch.randint(0, 4000, (t,), device=cuda, dtype=torch.int32)
    slot = torch.randperm(3 * 64, device=cuda)[:t].int()
    slot[5] = -1
    pool = torch.zeros(3, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8, device=cuda)
    pool_ref = pool.cpu().clone()
    ks, vs = (0.5, 0.25) if fmt == K.FMT_FP8 else (1.0, 1.0)
    q = K.gqa_prep(qkv, qn, kn, cs, pos, slot, pool, fmt, hq, hk, d, 1e-6, True, ks, vs)
    q_ref = K.gqa_prep(qkv.cpu(), qn.cpu(), kn.cpu(), cs.cpu(), pos.cpu(), slot.cpu(), pool_ref, fmt, hq, hk, d,
                       1e-6, True, ks, vs)
    assert torch.allclose(q.cpu().float(), q_ref.float(), rtol=1e-2, atol=1e-2)
    mism = (pool.cpu() != pool_ref).sum().item()
    # rope in fp32 may differ by one bf16 ulp -> rare single-code differences; require near bit-exactness
    assert mism <= max(4, pool.numel() // 20000), mism


def test_mla_and_index_writers_bitexact(cuda):
    torch.manual_seed(4)
    t = 33
    nope = (torch.randn(t, 512, device=cuda) * 3).to(torch.bfloat16)
    rope = torch.randn(t, 64, device=cuda).to(torch.bfloat16)
    slot = torch.randperm(100, device=cuda)[:t].int()
    for width in (352, 576):
        pool = torch.zeros(100, width, dtype=torch.uint8, device=cuda)
        ref = pool.cpu().clone()
        K.mla_write(nope, rope, slot, pool)
        K.mla_write(nope.cpu(), rope.cpu(), slot.cpu(), ref)
        assert torch.equal(pool.cpu(), ref), width
    k = torch.randn(t, 128, device=cuda).to(torch.bfloat16)
    pool = torch.zeros(2, K.INDEX_PAGE_BYTES, dtype=torch.uint8, device=cuda)
    ref = pool.cpu().clone()
    K.index_key_write(k, slot, pool)
    K.index_key_write(k.cpu(), slot.cpu(), ref)
    assert torch.equal(pool.cpu(), ref)
    assert torch.equal(K.index_key_read(ref, slot.cpu()), F.index_key_quantize(k.cpu()))


def _build_pool(cuda, fmt, d, hk, lens, scale=(1.0, 1.0), seed=0):
    torch.manual_seed(seed)
    b = len(lens)
    max_pages = max((n + 63) // 64 for n in lens)
    n_pages = b * max_pages + 3
    perm = torch.randperm(n_pages)
    pt = perm[: b * max_pages].reshape(b, max_pages).int()
    pool = torch.zeros(n_pages, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8)
    for i, n in enumerate(lens):
        k = torch.randn(n, hk, d).to(torch.bfloat16).float()
        v = torch.randn(n, hk, d).to(torch.bfloat16).float()
        pos = torch.arange(n)
        slot = pt[i][pos // 64].long() * 64 + pos % 64
        K.gqa_pool_write_ref(pool, slot, k, v, fmt, *scale)
    return pool.to(cuda), pt.to(cuda), torch.tensor(lens, dtype=torch.int32, device=cuda)


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("fmt", [K.FMT_NVFP4, K.FMT_FP8, K.FMT_BF16])
@pytest.mark.parametrize("d,window,n_q", [(512, 0, 1), (256, 96, 1), (512, 0, 4), (256, 0, 4), (128, 0, 1)])
def test_gqa_decode(cuda, fmt, d, window, n_q, exact):
    hq, hk = 4, 2
    lens = [300, 1, 129, 700][: 4] if n_q == 1 else [300, 4, 129, 700]
    scale = (0.5, 0.25) if fmt == K.FMT_FP8 else (1.0, 1.0)
    pool, pt, kv_len = _build_pool(cuda, fmt, d, hk, lens, scale)
    q = torch.randn(len(lens) * n_q, hq, d, device=cuda).to(torch.bfloat16)
    sm = 1.0 / math.sqrt(d)
    ref = A.gqa_decode_ref(q.cpu(), pool.cpu(), pt.cpu(), kv_len.cpu(), n_q, hk, fmt, sm, window, *scale)
    # E4M3 operands round K/V/Q/P once each (relative 2^-4): compare against the output's scale
    tol = 2e-2 if (exact or fmt == K.FMT_BF16) else 0.06 * max(1.0, ref.abs().max().item())
    for splits in (None, (1, 64)):
        out = A.gqa_decode(q, pool, pt, kv_len, n_q, hk, fmt, sm, window, *scale, splits=splits, exact=exact)
        torch.cuda.synchronize()
        err = (out.cpu().float() - ref).abs().max().item()
        assert err < tol, (splits, err)


def test_gqa_decode_long_context_splits(cuda):
    hq, hk, d = 4, 2, 512
    lens = [5000, 3333]
    pool, pt, kv_len = _build_pool(cuda, K.FMT_NVFP4, d, hk, lens, seed=7)
    q = torch.randn(2, hq, d, device=cuda).to(torch.bfloat16)
    sm = 1.0 / math.sqrt(d)
    ref = A.gqa_decode_ref(q.cpu(), pool.cpu(), pt.cpu(), kv_len.cpu(), 1, hk, K.FMT_NVFP4, sm)
    out = A.gqa_decode(q, pool, pt, kv_len, 1, hk, K.FMT_NVFP4, sm, exact=True)
    torch.cuda.synchronize()
    assert (out.cpu().float() - ref).abs().max().item() < 2e-2
    fast = A.gqa_decode(q, pool, pt, kv_len, 1, hk, K.FMT_NVFP4, sm)
    torch.cuda.synchronize()
    assert (fast.cpu().float() - ref).abs().max().item() < 0.06 * max(1.0, ref.abs().max().item())
    # deterministic
    out2 = A.gqa_decode(q, pool, pt, kv_len, 1, hk, K.FMT_NVFP4, sm)
    assert torch.equal(fast, out2)


def _mla_case(cuda, t, h, topk, fmt, rows=3000, mask_frac=0.1, seed=5):
    from inference_optimizations_b200.ops import mla as M
    torch.manual_seed(seed)
    nope = torch.randn(rows, 512)
    rope = torch.randn(rows, 64)
    pool = (F.mla_row_quantize(nope, rope) if fmt == K.FMT_NVFP4 else F.glmflash_row_quantize(nope) if fmt == 3
            else F.v4pro_cell_quantize(torch.cat([nope[:, :F.V4P_NOPE], rope], 1)) if fmt == 4
            else F.v4pro_cell_quantize(torch.cat([nope[:, :F.V4P_NOPE], rope], 1), "bf16") if fmt == 5
            else F.mla_fp8_row_quantize(nope, rope)).to(cuda)
    idx = torch.stack([torch.randperm(rows)[:topk] for _ in range(t)]).int()
    idx[torch.rand(t, topk) < mask_frac] = -1
    q = (torch.randn(t, h, 576) * 2).to(torch.bfloat16).to(cuda)
    q[:, :, 100] = 12.0              # one large channel: exercises the per-head query scale
    return M, pool, idx.to(cuda), q


@pytest.mark.parametrize("fmt", [K.FMT_NVFP4, K.FMT_FP8, 3, 4, 5])   # 3: rope-free 288-B row, 4 / 5: V4 Pro
                                                                    # 320-B (E4M3 rope) / 384-B (bf16 rope) cell
@pytest.mark.parametrize("t,h,topk", [(3, 128, 2048), (5, 64, 200), (2, 16, 64), (1, 128, 640)])
def test_mla_decode(cuda, fmt, t, h, topk):
    M, pool, idx, q = _mla_case(cuda, t, h, topk, fmt)
    sm = 1.0 / math.sqrt(576)
    ntiles = -(-topk // M.TILE)
    for splits in (None, (1, ntiles), (ntiles, 1)):
        sp = splits or M.mla_split_policy(t, topk)
        # against a CPU emulation of the E4M3 arithmetic and the same split schedule
        emu, emu_lse = M.mla_decode_emul_e4m3(q, pool, idx, sm, fmt, tiles_per_split=sp[1])
        out, lse = M.mla_decode(q, pool, idx, sm, fmt, splits=splits, return_lse=True)
        torch.cuda.synchronize()
        err = (out.float() - emu).abs().max().item()
        assert err < 2e-2 * max(1.0, emu.abs().max().item()), (splits, err)
        assert (lse - emu_lse).abs().max().item() < 2e-3, splits
    # and the E4M3 result stays within the rounding bound of the fp32 oracle
    ref, ref_lse = M.mla_decode_ref(q, pool, idx, sm, fmt)
    assert (out.float() - ref).abs().max().item() < 0.15 * max(1.0, ref.abs().max().item())
    assert (lse - ref_lse).abs().max().item() < 0.2


def test_mla_decode_masked_and_deterministic(cuda):
    M, pool, idx, q = _mla_case(cuda, 4, 128, 512, K.FMT_NVFP4, seed=9)
    idx[1] = -1                      # every row masked: zero output, -inf lse
    idx[2, 128:] = -1                # only the first tile visible
    sm = 1.0 / math.sqrt(576)
    ref, ref_lse = M.mla_decode_emul_e4m3(q, pool, idx, sm, K.FMT_NVFP4)
    out, lse = M.mla_decode(q, pool, idx, sm, K.FMT_NVFP4, splits=(1, 8), return_lse=True)
    out2 = M.mla_decode(q, pool, idx, sm, K.FMT_NVFP4, splits=(1, 8))
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    assert out[1].abs().max().item() == 0 and torch.isinf(lse[1]).all()
    assert (out.float() - ref).abs().max().item() < 2e-2 * max(1.0, ref.abs().max().item())
    assert (lse[[0, 2, 3]] - ref_lse[[0, 2, 3]]).abs().max().item() < 2e-3


@pytest.mark.parametrize("hi,topk", [(64, 2048), (32, 256)])
def test_indexer_scores_and_topk(cuda, hi, topk):
    from inference_optimizations_b200._ext import ext
    from inference_optimizations_b200.ops import indexer as I
    torch.manual_seed(11)
    lens = [300, 5000, 64, 2100, 1, 0]
    t = len(lens)
    per = max(-(-n // 64) for n in lens)
    pages = t * per + 2
    pt = torch.randperm(pages)[: t * per].view(t, per).int()
    pool = torch.zeros(pages, K.INDEX_PAGE_BYTES, dtype=torch.uint8)
    for i, n in enumerate(lens):
        if n:
            pos = torch.arange(n)
            K.index_key_write(torch.randn(n, 128).to(torch.bfloat16), (pt[i][pos // 64] * 64 + pos % 64).int(), pool)
    q8, w = I.indexer_q_quant(torch.randn(t, hi, 128), torch.rand(t, hi))
    limit = torch.tensor(lens, dtype=torch.int32)
    max_ctx = max(lens)
    ref = I.indexer_scores_ref(q8, w, pool, pt, limit, -(-max_ctx // 128) * 128)
    ws = I.IndexerWorkspace.allocate(t, max_ctx, cuda)
    slots, pos = I.indexer_select(q8.to(cuda), w.to(cuda), pool.to(cuda), pt.to(cuda), limit.to(cuda), topk,
                                  max_ctx, ws=ws, tiles_per_cta=8, with_pos=True)
    torch.cuda.synchronize()
    assert ws.status.item() == 0
    got = ws.scores.cpu()
    for i, n in enumerate(lens):
        if n:
            assert torch.allclose(got[i, :n], ref[i, :n], rtol=1e-4, atol=1e-4), i
    # selection is exact against the oracle run on the kernel's own scores
    rs, rp = I.topk_ref(got, limit, topk, pt)
    assert torch.equal(pos.cpu(), rp) and torch.equal(slots.cpu(), rs)


@pytest.mark.parametrize("fmt", [K.FMT_NVFP4, K.FMT_FP8])
@pytest.mark.parametrize("d,window", [(512, 0), (256, 96), (256, 0), (512, 200)])
def test_gqa_extend(cuda, fmt, d, window):
    """Prefill blocks (with a cached prefix, several requests, a partial last block) against the fp32 oracle."""
    hq, hk = 4, 2
    lens = [300, 77, 700]          # tokens in the pool per request; the last `new` of each are the query tokens
    new = [300, 77, 150]           # request 0: prefill from position 0; request 2: 550-token prefix
    scale = (0.5, 0.25) if fmt == K.FMT_FP8 else (1.0, 1.0)
    pool, pt, _ = _build_pool(cuda, fmt, d, hk, lens, scale, seed=3)
    segs, r0 = [], 0
    for i, (n, m) in enumerate(zip(lens, new)):
        segs.append((r0, m, n - m, i))
        r0 += m + 5                # gaps: rows outside every block stay untouched
    q = torch.randn(r0, hq, d, device=cuda).to(torch.bfloat16)
    blocks = torch.tensor(A.extend_blocks(segs, hq // hk), dtype=torch.int32, device=cuda)
    sm = 1.0 / math.sqrt(d)
    out = torch.full_like(q, 7.0)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    A.gqa_extend(q, pool, pt, blocks, hk, fmt, sm, window, *scale, out=out, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = A.gqa_extend_ref(q.cpu(), pool.cpu(), pt.cpu(), blocks.cpu(), hk, fmt, sm, window, *scale,
                           out=torch.full(q.shape, 7.0))
    tol = 0.06 * max(1.0, ref.abs().max().item())
    err = (out.cpu().float() - ref).abs().max().item()
    assert err < tol, err
    # the decode kernel over the same tokens (n_q = 1 per token) agrees to the same tolerance
    for s0, m, p0, i in segs[2:]:
        kvl = torch.arange(p0 + 1, p0 + m + 1, dtype=torch.int32, device=cuda)
        rix = torch.full((m,), i, dtype=torch.int32, device=cuda)
        dec = A.gqa_decode(q[s0:s0 + m].contiguous(), pool, pt, kvl, 1, hk, fmt, sm, window, *scale, req_idx=rix)
        torch.cuda.synchronize()
        assert (dec.float() - out[s0:s0 + m].float()).abs().max().item() < tol


@pytest.mark.parametrize("width", [9216, 20480, 70016, 204800, 262144, 300032])
def test_indexer_topk_ties_every_form(cuda, width):
    """Top-k selection alone over score rows with many exact ties (the one-CTA register form for rows up to 16384
    positions, the cluster form of 1 to 8 CTAs up to 262,144, the re-reading form beyond): the same positions, in
    position order, as the oracle."""
    from inference_optimizations_b200._ext import ext
    from inference_optimizations_b200.ops import indexer as I
    torch.manual_seed(2)
    lens = [width, width - 37, 3000, 2048, 1]
    t, topk = len(lens), 2048
    per = -(-width // 64)
    pt = torch.randperm(t * per + 1)[: t * per].view(t, per).int()
    scores = (torch.randn(t, width) * 4).round() / 4                  # few distinct values: ties at the threshold
    limit = torch.tensor(lens, dtype=torch.int32)
    slots = torch.empty(t, topk, dtype=torch.int32, device=cuda)
    pos = torch.empty(t, topk, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    q8 = torch.zeros(t, 64, 128, dtype=torch.uint8, device=cuda)
    w = torch.zeros(t, 64, device=cuda)
    pool = torch.zeros(1, K.INDEX_PAGE_BYTES, dtype=torch.uint8, device=cuda)
    sc = scores.to(cuda)
    ext().indexer(q8, w, pool, pt.to(cuda), None, limit.to(cuda), sc, slots, pos, status, 1, width // 128, 0, 1)
    torch.cuda.synchronize()
    rs, rp = I.topk_ref(scores, limit, topk, pt)
    assert torch.equal(pos.cpu(), rp) and torch.equal(slots.cpu(), rs)
