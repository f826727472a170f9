"""Fused KDA decode kernel (csrc/kda.cu) against the fp32 oracle over several steps (state carried)."""
import pytest
import torch

from inference_optimizations_b200.ops import kda as KD

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("headwise,W", [(False, 4), (True, 4), (False, 2)])
def test_kda_decode_matches_oracle(cuda, headwise, W):
    from test_kda_cpu import _inputs
    a = _inputs(B=3, H=4, W=W, seed=7, headwise=headwise)
    g = {k: v.to(cuda).contiguous() for k, v in a.items()}
    r = {k: v.clone() for k, v in a.items()}
    for step in range(4):
        o = KD.kda_decode(**g)
        o_ref = KD.kda_decode_ref(**r)
        torch.cuda.synchronize()
        assert torch.allclose(o.float().cpu(), o_ref.float(), atol=3e-2, rtol=3e-2), (step, (o.float().cpu() - o_ref.float()).abs().max())
        assert torch.allclose(g["state"].cpu(), r["state"], atol=1e-4, rtol=1e-3)
        assert torch.allclose(g["csv"].cpu(), r["csv"])
        # next token's projections
        for k in ("q", "k", "v", "g_proj", "g2"):
            nv = torch.randn_like(r[k].float()).to(r[k].dtype)
            r[k], g[k] = nv, nv.to(cuda)


@pytest.mark.parametrize("m", [4096, 120, 24])
def test_small_projection_fuse_gpu(m):
    """Fused (one GEMM + one bmm) vs separate (five GEMMs) KDA small projections: equal within a bf16 ulp; prints the
    CUDA-graph replay time of both."""
    from inference_optimizations_b200.ops.kda import KDASmallProjections
    torch.manual_seed(0)
    H, nb, d, P = 2048, 32, 128, 4096
    ws = [torch.randn(s, device="cuda", dtype=torch.bfloat16) * 0.03 for s in ((nb, H), (d, H), (P, d), (d, H),
                                                                                 (P, d))]
    sp = KDASmallProjections(*ws)
    x = torch.randn(m, H, device="cuda", dtype=torch.bfloat16)

    def graph_us(fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(50):
            g.replay()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / 50, out

    t_sep, ref = graph_us(lambda: sp.forward_separate(x))
    ref = [r.clone() for r in ref]
    sp.fuse()
    t_fused, out = graph_us(lambda: sp.forward(x))
    for a, b in zip(ref, out):
        ulp = a.float().abs().clamp_min(1e-3) * 2 ** -7
        assert ((a.float() - b.float()).abs() <= ulp).all()
    print(f"KDA small projections M={m}: separate {t_sep:.1f} us, fused {t_fused:.1f} us")
