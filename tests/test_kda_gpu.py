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
