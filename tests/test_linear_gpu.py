"""Projection GEMMs of the MLA family on the tcgen05 weight-streaming kernels, each against a plain fp32 PyTorch
reference of the same op: head-batched bf16 products read in place from a wider projection output, padded FP8 / bf16
linears with odd widths, the fp32-output router GEMM, the streaming (one expert at a time) expert build, and the MLA
model whose every projection runs on these kernels."""
import pytest
import torch

from inference_optimizations_b200.ops import linear as L
from inference_optimizations_b200.ops import moe_gemm as MG

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t,H,N,K,stride", [(1, 128, 512, 128, 256), (37, 128, 512, 128, 256),
                                             (200, 128, 128, 512, 0), (5, 64, 512, 192, 107)])
def test_head_batched_linear(cuda, t, H, N, K, stride):
    torch.manual_seed(t + N)
    w = (torch.randn(H, N, K, device=cuda) * 0.05).to(torch.bfloat16)
    rs = stride or H
    buf = torch.randn(t, rs * K, device=cuda).to(torch.bfloat16)          # head h of token t at row t * rs + h
    x = buf.view(t, rs, K)[:, :H]
    hb = L.HeadBatchedLinear(w)
    y = hb(buf, t, row_stride=stride)
    ref = torch.einsum("thk,hnk->thn", x.float(), w.float())
    assert y.shape == (t, H, N)
    err = (y.float() - ref).abs().max().item()
    assert err < 2e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("kind", ["fp8", "bf16"])
@pytest.mark.parametrize("t,N,K", [(3, 2304, 7168), (64, 836, 256), (300, 640, 1536)])
def test_padded_linear(cuda, kind, t, N, K):
    torch.manual_seed(N)
    w = (torch.randn(N, K, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(t, K, device=cuda).to(torch.bfloat16)
    lin = L.Linear(w, kind)
    y = lin(x)
    assert y.shape == (t, N)
    if kind == "fp8":
        wq, we = MG.quant_blocks(torch.cat([w, torch.zeros(lin.Np - N, K, device=cuda, dtype=w.dtype)])[None])
        wd = MG.dequant_blocks(wq, we)[0][:N]
        xd = MG.dequant_rows(*MG.quant_rows(x.float()))
        ref = xd @ wd.t()
    else:
        ref = x.float() @ w.float().t()
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 1e-2, rel.item()


def test_fused_linear_split(cuda):
    torch.manual_seed(2)
    ws = [(torch.randn(n, 512, device=cuda) * 0.02).to(torch.bfloat16) for n in (128, 64, 100)]
    x = torch.randn(9, 512, device=cuda).to(torch.bfloat16)
    lin = L.Linear.fuse(ws, "bf16")
    parts = lin.split(lin(x))
    for w, p in zip(ws, parts):
        ref = x.float() @ w.float().t()
        assert p.shape == (9, w.shape[0])
        assert (p.float() - ref).abs().max().item() < 2e-2


def test_router_logits_fp32(cuda):
    torch.manual_seed(3)
    w = (torch.randn(256, 7168, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(33, 7168, device=cuda).to(torch.bfloat16)
    y = L.Linear(w, "bf16")(x, out_f32=True)
    assert y.dtype == torch.float32
    ref = x.float() @ w.float().t()
    assert (y - ref).abs().max().item() < 1e-3


@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
def test_streaming_expert_build_matches_stacked(cuda, fmt):
    torch.manual_seed(4)
    E, F, H = 3, 256, 512
    g = (torch.randn(E, F, H, device=cuda) * 0.02).to(torch.bfloat16)
    u = (torch.randn(E, F, H, device=cuda) * 0.02).to(torch.bfloat16)
    d = (torch.randn(E, H, F, device=cuda) * 0.02).to(torch.bfloat16)
    sh = ((torch.randn(F, H, device=cuda) * 0.02).to(torch.bfloat16),
          (torch.randn(F, H, device=cuda) * 0.02).to(torch.bfloat16),
          (torch.randn(H, F, device=cuda) * 0.02).to(torch.bfloat16))
    a = MG.BlockScaledExperts(g, u, d, shared=sh, fmt=fmt)
    b = MG.BlockScaledExperts.build(10, 10 + E, F, H, lambda e: (g[e - 10], u[e - 10], d[e - 10]), shared=sh,
                                    fmt=fmt, device=cuda)
    assert torch.equal(a.w1, b.w1) and torch.equal(a.w2, b.w2)
    if fmt == "nvfp4":
        assert torch.equal(a.mul1, b.mul1) and torch.equal(a.mul2, b.mul2)


def test_mla_model_fp8_projections_track_bf16(cuda):
    """The MLA model with FP8 block-scaled projections (every GEMM on the tcgen05 kernels) stays close to its bf16
    twin run by the torch reference path on the same weights."""
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import Request, SamplingParams, Segment
    over = dict(expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8", hidden=512, q_lora=256,
                qk_nope=128, v_head=128)
    cfg = model_config("tiny_mla", **over)
    ecfg = EngineConfig(model="tiny_mla", device=str(cuda), kv_dtype="fp8", max_running=4, chunked_prefill=64,
                        cuda_graphs=False, prefix_cache=False)
    gpu = Engine(ecfg, cfg, max_seq=256)
    assert gpu.runner.model.layers[0].k is not None and "uk" in gpu.runner.model.layers[0].k
    cpu = Engine(EngineConfig(**dict(vars(ecfg), device="cpu")), cfg, max_seq=256)
    cpu.runner.model.copy_from(gpu.runner.model)
    torch.manual_seed(5)
    prompt = torch.randint(0, cfg.vocab, (70,)).tolist()
    logits = []
    for eng in (gpu, cpu):
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        logits.append(eng.runner.model.logits(eng.runner.model.forward(st, eng.runner.kv)).float().cpu())
    cos = torch.nn.functional.cosine_similarity(logits[0], logits[1], dim=-1)
    assert cos.mean().item() > 0.97 and cos.min().item() > 0.85, (cos.mean().item(), cos.min().item())


@pytest.mark.parametrize("kv", ["nvfp4", "fp8"])
def test_mla_fused_glue_matches_torch_glue(cuda, kv):
    """The two fused glue kernels (norms, RoPE, pool writes, indexer query quantization) reproduce the torch glue of
    the same layer: same latent / index pool bytes up to rounding flips, logits within bf16 noise."""
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import Request, SamplingParams, Segment
    over = dict(expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8", hidden=512, q_lora=256,
                qk_nope=128, v_head=128, index_heads=8, num_heads=8)
    cfg = model_config("tiny_mla", **over)
    ecfg = EngineConfig(model="tiny_mla", device=str(cuda), kv_dtype=kv, max_running=4, chunked_prefill=128,
                        cuda_graphs=False, prefix_cache=False)
    torch.manual_seed(6)
    prompt = torch.randint(0, cfg.vocab, (100,)).tolist()
    res = []
    for fused in (False, True):
        eng = Engine(ecfg, cfg, max_seq=256)
        eng.runner.model.fuse_glue = fused
        assert eng.runner.model._fused_glue(eng.runner.model.layers[0]) == fused
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        logits = eng.runner.model.logits(eng.runner.model.forward(st, eng.runner.kv)).float()
        torch.cuda.synchronize()
        res.append((logits.cpu(), [p.clone().cpu() for p in eng.runner.kv.latent],
                    [p.clone().cpu() for p in eng.runner.kv.index]))
    (l0, lat0, idx0), (l1, lat1, idx1) = res
    for a, b in zip(lat0 + idx0, lat1 + idx1):
        assert (a != b).float().mean().item() < 0.01          # a few rounding-boundary flips at most
    cos = torch.nn.functional.cosine_similarity(l0, l1, dim=-1)
    assert cos.min().item() > 0.999, cos.min().item()


@pytest.mark.parametrize("kind,t", [("fp8", 8), ("fp8", 64), ("bf16", 8)])
def test_folded_splitk_equals_separate_reduction(cuda, kind, t):
    """The split-K reduction folded into the GEMM (the split completing a tile sums the partials) gives the separate
    reduction kernel's bits, on repeated calls (the tile counters re-arm) and for fp32 output."""
    torch.manual_seed(t)
    w = (torch.randn(7168, 16384, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(t, 16384, device=cuda).to(torch.bfloat16)
    lin = L.Linear(w, kind)
    ref = lin(x).clone()
    fold_max, L.FOLD_MAX_TOKENS = L.FOLD_MAX_TOKENS, 1 << 20      # fold at every token count for this test
    L.FOLD_SPLITK[0] = True
    try:
        for _ in range(3):
            assert torch.equal(lin(x), ref)
    finally:
        L.FOLD_MAX_TOKENS = fold_max
        L.FOLD_SPLITK[0] = False
    if kind == "bf16":
        ref32 = lin(x, out_f32=True).clone()
        L.FOLD_SPLITK[0] = True
        try:
            assert torch.equal(lin(x, out_f32=True), ref32)
        finally:
            L.FOLD_SPLITK[0] = False


def test_rmsnorm_fp8_output_equals_separate_quant(cuda):
    """RMSNorm (+ residual) writing the FP8 block-scaled copy gives the bytes of quantizing its bf16 output with the
    activation-quantization kernel afterwards."""
    from inference_optimizations_b200._ext import ext
    from inference_optimizations_b200.ops import basic as B
    torch.manual_seed(9)
    t, h = 37, 7168
    x = torch.randn(t, h, device=cuda).to(torch.bfloat16)
    res = torch.randn(t, h, device=cuda).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(h, device=cuda)).to(torch.bfloat16)
    res2 = res.clone()
    q8 = torch.empty(t, h, dtype=torch.uint8, device=cuda)
    qs = torch.empty(t, h // 128, dtype=torch.int32, device=cuda)
    y = B.rmsnorm(x, w, 1e-6, residual=res, fp8=(q8, qs))
    y_ref = B.rmsnorm(x, w, 1e-6, residual=res2)
    rq = torch.empty_like(q8)
    rs = torch.empty_like(qs)
    ext().rmsnorm_quant(y_ref, None, 0.0, 0.0, rq, rs, 0)
    assert torch.equal(y, y_ref) and torch.equal(res, res2)
    assert torch.equal(q8, rq) and torch.equal(qs, rs)
