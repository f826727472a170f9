"""Block-scaled grouped expert GEMM (tcgen05 kind::mxf8f6f4) and the FP8 MoE feed-forward against fp32 oracles."""
import pytest
import torch
import torch.nn.functional as Fn

from inference_optimizations_b200.ops import moe_gemm as MG

pytestmark = pytest.mark.gpu


def _case(cuda, E, N, K, T, topk, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, N, K, generator=g)
    # per-row weight scales spread over 2^-6 .. 2^6 exercise the A scale-factor layout row by row
    w = w * torch.exp2(torch.randint(-6, 7, (E, N, 1), generator=g).float())
    x = torch.randn(T, K, generator=g) * torch.exp2(torch.randint(-8, 9, (T, 1), generator=g).float())
    ids = torch.randint(0, E, (T, topk), generator=g, dtype=torch.int32)
    return w, x, ids


def _quant_rowwise_weights(w):
    E, N, K = w.shape
    q, sc = MG.quant_rows(w.reshape(E * N, K))
    return q.view(E, N, K), (sc & 0xFF).to(torch.uint8).view(E, N, K // 128), MG.dequant_rows(q, sc).view(E, N, K)


@pytest.mark.parametrize("nt", [16, 32, 64, 128])
@pytest.mark.parametrize("ctas", [148, 3])
def test_moe_gemm_plain(cuda, nt, ctas):
    from inference_optimizations_b200._ext import ext
    E, N, K, T, topk = 3, 256, 384, 37, 2
    w, x, ids = _case(cuda, E, N, K, T, topk, seed=nt + ctas)
    wq, web, wd = _quant_rowwise_weights(w)
    xq, xs = MG.quant_rows(x)
    xd = MG.dequant_rows(xq, xs)
    pack = MG.pack_weights([wq], [web]).to(cuda)
    P = T * topk
    off = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    pairs = torch.empty(P, dtype=torch.int32, device=cuda)
    ext().moe_align(ids.view(-1).to(cuda), 0, E, 0, off, pairs)
    cnt = torch.bincount(ids.view(-1).long(), minlength=E)
    assert off.cpu().tolist() == [0] + torch.cumsum(cnt, 0).tolist()
    out = torch.zeros(P, N, dtype=torch.bfloat16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    MG.gemm(pack, xq.to(cuda), xs.to(cuda), off, pairs, out, status, n_tiles=N // 128, kc=K // 128, g=1, nt=nt,
            mode=0, src_div=topk, src_limit=P, num_ctas=ctas)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = torch.stack([xd[p // topk] @ wd[int(ids.view(-1)[p])].T for p in range(P)])
    got = out.float().cpu()
    err = (got - ref).abs() / (ref.abs() + 1e-3 * ref.abs().amax(1, keepdim=True))
    assert err.max().item() < 1e-2, err.max().item()


@pytest.mark.parametrize("nt", [16, 64])
def test_moe_gemm_swiglu_quant(cuda, nt):
    from inference_optimizations_b200._ext import ext
    E, F, K, T, topk = 2, 256, 256, 20, 2
    g = torch.Generator().manual_seed(7)
    wg = torch.randn(E, F, K, generator=g) * 0.05
    wu = torch.randn(E, F, K, generator=g) * 0.05
    x = torch.randn(T, K, generator=g)
    ids = torch.randint(0, E, (T, topk), generator=g, dtype=torch.int32)
    qg, eg = MG.quant_blocks(wg)
    qu, eu = MG.quant_blocks(wu)
    pack = MG.pack_weights([qg, qu], [eg, eu]).to(cuda)
    xq, xs = MG.quant_rows(x)
    xd = MG.dequant_rows(xq, xs)
    P = T * topk
    off = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    pairs = torch.empty(P, dtype=torch.int32, device=cuda)
    ext().moe_align(ids.view(-1).to(cuda), 0, E, 0, off, pairs)
    h = torch.zeros(P, F, dtype=torch.uint8, device=cuda)
    hs = torch.zeros(P, F // 128, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    MG.gemm(pack, xq.to(cuda), xs.to(cuda), off, pairs, h, status, n_tiles=F // 128, kc=K // 128, g=2, nt=nt,
            mode=1, src_div=topk, src_limit=P, out_scale=hs)
    torch.cuda.synchronize()
    assert status.item() == 0
    dg, du = MG.dequant_blocks(qg, eg), MG.dequant_blocks(qu, eu)
    e_of = ids.view(-1).long()
    hh = torch.stack([Fn.silu(xd[p // topk] @ dg[e_of[p]].T) * (xd[p // topk] @ du[e_of[p]].T) for p in range(P)])
    rq, rs = MG.quant_rows(hh)
    # scales: the same power of two except where amax sits within float rounding of a boundary
    assert ((hs.cpu() & 0xFF) == (rs & 0xFF)).float().mean().item() > 0.97
    got = MG.dequant_rows(h.cpu(), hs.cpu())
    cos = Fn.cosine_similarity(got.flatten(), hh.flatten(), dim=0).item()
    assert cos > 0.998, cos
    assert (h.cpu() == rq).float().mean().item() > 0.95


def test_rmsnorm_quant_matches_oracle(cuda):
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(3)
    x = (torch.randn(6, 512) * torch.exp2(torch.randint(-5, 6, (6, 1)).float())).to(torch.bfloat16)
    q = torch.empty(6, 512, dtype=torch.uint8, device=cuda)
    sc = torch.empty(6, 4, dtype=torch.int32, device=cuda)
    ext().rmsnorm_quant(x.to(cuda), None, 0.0, 0.0, q, sc, 0)
    rq, rs = MG.quant_rows(x.float())
    assert torch.equal(sc.cpu(), rs) and torch.equal(q.cpu(), rq)
    w = (torch.randn(512) * 0.1).to(torch.bfloat16)
    ext().rmsnorm_quant(x.to(cuda), w.to(cuda), 1e-6, 1.0, q, sc, 0)
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * (w.float() + 1.0)).to(torch.bfloat16).float()
    rq, rs = MG.quant_rows(n)
    assert (q.cpu() == rq).float().mean().item() > 0.99
    assert torch.equal(sc.cpu(), rs)


@pytest.mark.parametrize("shared", [False, True])
def test_fp8_experts_forward(cuda, shared):
    torch.manual_seed(11)
    E, F, H, T, topk = 6, 256, 512, 13, 3
    wg = torch.randn(E, F, H, device=cuda) * 0.04
    wu = torch.randn(E, F, H, device=cuda) * 0.04
    wd = torch.randn(E, H, F, device=cuda) * 0.04
    sh = tuple(torch.randn(*s, device=cuda) * 0.04 for s in ((F, H), (F, H), (H, F))) if shared else None
    ex = MG.Fp8Experts(wg, wu, wd, shared=sh)
    x = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device=cuda)[:topk] for _ in range(T)]).int()
    w = torch.softmax(torch.randn(T, topk, device=cuda), -1)
    y = ex.forward(x, ids, w)
    torch.cuda.synchronize()
    assert ex.status.item() == 0
    ref = ex.forward_ref(x, ids, w)
    cos = Fn.cosine_similarity(y.float().flatten(), ref.float().flatten(), dim=0).item()
    assert cos > 0.999, cos
    rel = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel < 0.03, rel


def test_moe_gemm_paired_tiles(cuda):
    """Plain output with two adjacent 128-column tiles per CTA (G = 2) equals the single-tile launch."""
    from inference_optimizations_b200._ext import ext
    E, N, K, T, topk = 2, 512, 256, 19, 2
    w, x, ids = _case(cuda, E, N, K, T, topk, seed=5)
    wq, web, wd = _quant_rowwise_weights(w)
    xq, xs = MG.quant_rows(x)
    P = T * topk
    off = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    pairs = torch.empty(P, dtype=torch.int32, device=cuda)
    ext().moe_align(ids.view(-1).to(cuda), 0, E, 0, off, pairs)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = []
    for pack, g in (MG.pack_weights_paired(wq, web), (MG.pack_weights([wq], [web]), 1)):
        out = torch.zeros(P, N, dtype=torch.bfloat16, device=cuda)
        MG.gemm(pack.to(cuda), xq.to(cuda), xs.to(cuda), off, pairs, out, status, n_tiles=N // (128 * g),
                kc=K // 128, g=g, nt=32, mode=0, src_div=topk, src_limit=P)
        outs.append(out)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("nt", [16, 128])
def test_moe_gemm_nvfp4_plain(cuda, nt):
    """kind::mxf4nvf4 (E2M1 x E2M1, E4M3 scale per 16): every scale byte differs, so the four scale atoms per
    chunk and their row layout are all exercised; the per-expert global scale comes in through expert_mul."""
    from inference_optimizations_b200._ext import ext
    E, N, K, T, topk = 3, 256, 512, 29, 2
    w, x, ids = _case(cuda, E, N, K, T, topk, seed=40 + nt)
    wq, ws, wg = MG.quant_nvfp4_weights(w)
    wd = MG.dequant_nvfp4_weights(wq, ws, wg)
    xq, xs = MG.quant_nvfp4_rows(x)
    xd = MG.dequant_nvfp4_rows(xq, xs)
    pack = MG.pack_weights_nvfp4([wq], [ws]).to(cuda)
    P = T * topk
    off = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    pairs = torch.empty(P, dtype=torch.int32, device=cuda)
    ext().moe_align(ids.view(-1).to(cuda), 0, E, 0, off, pairs)
    out = torch.zeros(P, N, dtype=torch.bfloat16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    MG.gemm(pack, xq.to(cuda), xs.to(cuda), off, pairs, out, status, n_tiles=N // 128, kc=K // 256, g=1, nt=nt,
            mode=0, src_div=topk, src_limit=P, kind=1, expert_mul=wg.to(cuda))
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = torch.stack([xd[p // topk] @ wd[int(ids.view(-1)[p])].T for p in range(P)])
    got = out.float().cpu()
    err = (got - ref).abs() / (ref.abs() + 1e-3 * ref.abs().amax(1, keepdim=True))
    assert err.max().item() < 1e-2, err.max().item()


def test_quant_nvfp4_rows_matches_oracle(cuda):
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(9)
    x = (torch.randn(5, 512) * torch.exp2(torch.randint(-5, 6, (5, 1)).float())).to(torch.bfloat16)
    q = torch.empty(5, 256, dtype=torch.uint8, device=cuda)
    sc = torch.empty(5, 8, dtype=torch.int32, device=cuda)
    ext().rmsnorm_quant(x.to(cuda), None, 0.0, 0.0, q, sc, 1)
    rq, rs = MG.quant_nvfp4_rows(x.float())
    assert torch.equal(q.cpu(), rq) and torch.equal(sc.cpu(), rs)


@pytest.mark.parametrize("shared", [False, True])
def test_nvfp4_experts_forward(cuda, shared):
    torch.manual_seed(12)
    E, F, H, T, topk = 5, 256, 512, 11, 2
    wg = torch.randn(E, F, H, device=cuda) * 0.04
    wu = torch.randn(E, F, H, device=cuda) * 0.04
    wd = torch.randn(E, H, F, device=cuda) * 0.04
    sh = tuple(torch.randn(*s, device=cuda) * 0.04 for s in ((F, H), (F, H), (H, F))) if shared else None
    ex = MG.BlockScaledExperts(wg, wu, wd, shared=sh, fmt="nvfp4")
    x = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device=cuda)[:topk] for _ in range(T)]).int()
    w = torch.softmax(torch.randn(T, topk, device=cuda), -1)
    y = ex.forward(x, ids, w)
    torch.cuda.synchronize()
    assert ex.status.item() == 0
    ref = ex.forward_ref(x, ids, w)
    cos = Fn.cosine_similarity(y.float().flatten(), ref.float().flatten(), dim=0).item()
    assert cos > 0.995, cos


@pytest.mark.parametrize("t,n,k", [(5, 384, 256), (32, 1024, 512), (77, 256, 192)])
def test_dense_bf16_linear(cuda, t, n, k):
    """kind::f16 weight-streaming GEMM (tokens as N) against an fp32 matmul of the same bf16 values."""
    from inference_optimizations_b200.ops.linear import DenseLinear
    torch.manual_seed(t)
    w = (torch.randn(n, k, device=cuda) * 0.05).to(torch.bfloat16)
    x = torch.randn(t, k, device=cuda).to(torch.bfloat16)
    lin = DenseLinear(w)
    y = lin(x)
    torch.cuda.synchronize()
    assert lin.status.item() == 0
    ref = x.float() @ w.float().T
    err = (y.float() - ref).abs() / (ref.abs() + 1e-2 * ref.abs().max())
    assert err.max().item() < 1e-2, err.max().item()


def test_fp8_linear_and_sharded_lm_head(cuda):
    from inference_optimizations_b200.ops.linear import Fp8Linear, ShardedLMHead
    torch.manual_seed(4)
    w = (torch.randn(1000, 512, device=cuda) * 0.05).to(torch.bfloat16)
    x = torch.randn(7, 512, device=cuda).to(torch.bfloat16)
    lin = Fp8Linear(w[:896])
    y = lin(x)
    xq, xs = MG.quant_rows(x.float())
    ref = MG.dequant_rows(xq, xs) @ lin.dequant().T
    err = (y.float() - ref).abs() / (ref.abs() + 1e-2 * ref.abs().max())
    assert err.max().item() < 1e-2
    # vocabulary-parallel head over 2 shards (same GPU): merged argmax equals the argmax of the full FP8 logits
    heads = [ShardedLMHead(w, r, 2) for r in range(2)]
    vals, ids = zip(*[h.local_argmax(x) for h in heads])
    v = torch.stack(vals, 1)
    i = torch.stack(ids, 1)
    best = i.gather(1, v.argmax(1, keepdim=True))[:, 0]
    full = torch.cat([h.lin(x)[:, :h.rows].float() for h in heads], 1)
    assert torch.equal(best, full.argmax(1))


@pytest.mark.parametrize("gelu", [True, False])
@pytest.mark.parametrize("fmt", [0, 1])
def test_act_quant_bitexact(cuda, gelu, fmt):
    """One-pass act(gate) * up + quant equals quantizing the bf16 act_mul output, bit for bit."""
    from inference_optimizations_b200.ops import basic as B
    from inference_optimizations_b200.ops.linear import act_quant
    torch.manual_seed(5)
    gu = (torch.randn(37, 2 * 1024, device=cuda) * 2).to(torch.bfloat16)
    q, s = act_quant(gu, gelu, fmt)
    a = B.act_mul(gu, gelu)
    rq, rs = MG.quant_rows(a) if fmt == 0 else MG.quant_nvfp4_rows(a)
    assert torch.equal(q, rq) and torch.equal(s, rs)


def test_fp8_mlp(cuda):
    from inference_optimizations_b200.ops.linear import Fp8Mlp
    torch.manual_seed(6)
    wgu = (torch.randn(2 * 768, 512, device=cuda) * 0.05).to(torch.bfloat16)
    wd = (torch.randn(512, 768, device=cuda) * 0.05).to(torch.bfloat16)
    x = torch.randn(9, 512, device=cuda).to(torch.bfloat16)
    mlp = Fp8Mlp(wgu, wd)
    y = mlp(x).float()
    ref = mlp.reference(x).to(y.device)
    err = (y - ref).abs() / (ref.abs() + 1e-2 * ref.abs().max())
    assert err.max().item() < 2e-2


@pytest.mark.parametrize("t,n,k", [(5, 256, 4096), (33, 384, 8192), (16, 5376, 21504)])
def test_dense_linear_split_k(cuda, t, n, k):
    """Split-K weight streaming (few output tiles, long K: fp32 partials per K range, one ordered reduction) against
    an fp32 matmul, and run to run identical."""
    from inference_optimizations_b200.ops.linear import DenseLinear, split_k
    import inference_optimizations_b200.ops.moe_gemm as MGm
    torch.manual_seed(t)
    w = (torch.randn(n, k, device=cuda) * 0.05).to(torch.bfloat16)
    x = torch.randn(t, k, device=cuda).to(torch.bfloat16)
    lin = DenseLinear(w)
    assert split_k(n // (128 * lin.g), t, MGm.pick_nt(t), k // 64, lin.num_ctas) > 1
    y = lin(x)
    y2 = lin(x)
    torch.cuda.synchronize()
    assert lin.status.item() == 0 and torch.equal(y, y2)
    ref = x.float() @ w.float().T
    err = (y.float() - ref).abs() / (ref.abs() + 1e-2 * ref.abs().max())
    assert err.max().item() < 1e-2, err.max().item()


@pytest.mark.parametrize("fmt", [0, 1])
def test_rmsnorm_quant_wide_rows_spread_over_ctas(cuda, fmt):
    """Few wide rows without a norm spread each row over several CTAs (the decode-size quantization of the o_proj
    input): the same bytes as the row-per-CTA oracle."""
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(5)
    T, H = 3, 16384
    x = (torch.randn(T, H) * torch.exp2(torch.randint(-5, 6, (T, H // 128)).float().repeat_interleave(128, 1)))
    x = x.to(torch.bfloat16)
    q = torch.empty(T, H if fmt == 0 else H // 2, dtype=torch.uint8, device=cuda)
    sc = torch.empty(T, H // 128 if fmt == 0 else H // 64, dtype=torch.int32, device=cuda)
    ext().rmsnorm_quant(x.to(cuda), None, 0.0, 0.0, q, sc, fmt)
    rq, rs = MG.quant_rows(x.float()) if fmt == 0 else MG.quant_nvfp4_rows(x.float())
    assert torch.equal(q.cpu(), rq) and torch.equal(sc.cpu(), rs)


def test_dense_ffn_split_down_projection(cuda):
    """A dense FFN (one expert holding every token) at decode sizes splits its down projection over K; the result
    matches the fp32 oracle, and a token's output does not depend on the batch it runs in (up to 64 tokens)."""
    torch.manual_seed(12)
    F, H = 4096, 1024
    wg = torch.randn(1, F, H, device=cuda) * 0.03
    wu = torch.randn(1, F, H, device=cuda) * 0.03
    wd = torch.randn(1, H, F, device=cuda) * 0.03
    ex = MG.Fp8Experts(wg, wu, wd)
    assert ex._dense_split(H // (128 * ex.g2), F // 128, 16) > 1
    x = torch.randn(9, H, device=cuda).to(torch.bfloat16)
    one = lambda n: (torch.zeros(n, 1, dtype=torch.int32, device=cuda), torch.ones(n, 1, device=cuda))  # noqa: E731
    y = ex.forward(x, *one(9))
    torch.cuda.synchronize()
    assert ex.status.item() == 0
    ref = ex.forward_ref(x, *one(9))
    cos = Fn.cosine_similarity(y.float().flatten(), ref.float().flatten(), dim=0).item()
    assert cos > 0.999, cos
    y3 = ex.forward(x[:3].contiguous(), *one(3))
    assert torch.equal(y3, y[:3])
