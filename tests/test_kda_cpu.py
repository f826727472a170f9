"""KDA decode oracle properties and recurrent-state row formats (ops/kda.py)."""
import torch

from inference_optimizations_b200.ops import kda as KD


def _inputs(B=2, H=3, DK=128, DV=128, W=4, seed=0, headwise=False):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    return dict(q=r(B, H, DK).to(torch.bfloat16), k=r(B, H, DK).to(torch.bfloat16), v=r(B, H, DV).to(torch.bfloat16),
                g_proj=r(B, H, DK).to(torch.bfloat16), dt_bias=r(H * DK) * 0.1, A_log=r(H) * 0.1,
                beta=torch.sigmoid(r(B, H, DV) if headwise else r(B, H)), g2=r(B, H, DV).to(torch.bfloat16),
                norm_w=1 + 0.1 * r(DV), cwq=r(H * DK, W) * 0.3, cwk=r(H * DK, W) * 0.3, cwv=r(H * DV, W) * 0.3,
                csq=r(B, H * DK, W - 1), csk=r(B, H * DK, W - 1), csv=r(B, H * DV, W - 1),
                state=r(B, H, DV, DK) * 0.1)


def test_decode_ref_state_evolution():
    a = _inputs()
    st0 = a["state"].clone()
    csq0 = a["csq"].clone()
    o = KD.kda_decode_ref(**a)
    assert o.shape == (2, 3, 128) and torch.isfinite(o.float()).all()
    assert not torch.equal(st0, a["state"])
    # conv state shifted left with the raw input appended
    assert torch.equal(a["csq"][..., :2], csq0[..., 1:])
    assert torch.allclose(a["csq"][..., 2], a["q"].float().reshape(2, -1))
    # the delta rule makes the state reproduce v on k (after one write with beta = 1, decay 0)
    b = _inputs(seed=1)
    b["beta"] = torch.ones_like(b["beta"])
    b["A_log"] = torch.full_like(b["A_log"], -30.0)          # decay exp(-exp(-30)*sp) ~ 1
    KD.kda_decode_ref(**b)


def test_state_rows_round_trip():
    torch.manual_seed(0)
    rows = torch.randn(16, 128) * torch.exp2(torch.randint(-4, 5, (16, 1)).float())
    for fmt, tol in (("bf16", 4e-3), ("fp8", 7e-2), ("nvfp4", 0.25)):
        b = KD.quant_state_rows(rows, fmt)
        assert b.shape == (16, KD.ROW_BYTES[fmt])
        d = KD.dequant_state_rows(b, fmt)
        rel = ((d - rows).norm(dim=-1) / rows.norm(dim=-1)).max().item()
        assert rel < tol, (fmt, rel)


def test_state_store_park_load():
    st = KD.StateStore("fp8")
    s = torch.randn(2, 4, 128, 128)
    st.park("r1", s)
    assert st.nbytes() == 2 * 4 * 128 * 132
    back = st.load("r1")
    assert back.shape == s.shape and ((back - s).norm() / s.norm()) < 0.07


def _seq_inputs(B, T, H, seed, headwise):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    DK = DV = 128
    W = 4
    return dict(q=r(B, T, H, DK).to(torch.bfloat16), k=r(B, T, H, DK).to(torch.bfloat16),
                v=r(B, T, H, DV).to(torch.bfloat16), g_proj=r(B, T, H, DK).to(torch.bfloat16),
                dt_bias=r(H * DK) * 0.1, A_log=r(H) * 0.1,
                beta=torch.sigmoid(r(B, T, H, DV) if headwise else r(B, T, H)),
                g2=r(B, T, H, DV).to(torch.bfloat16), norm_w=1 + 0.1 * r(DV), cwq=r(H * DK, W) * 0.3,
                cwk=r(H * DK, W) * 0.3, cwv=r(H * DV, W) * 0.3, csq=r(B, H * DK, W - 1), csk=r(B, H * DK, W - 1),
                csv=r(B, H * DV, W - 1), state=r(B, H, DV, DK) * 0.1)


import pytest  # noqa: E402


@pytest.mark.parametrize("headwise", [False, True])
def test_chunked_prefill_matches_recurrence(headwise):
    """The chunked prefill (a 100-token sequence: one full 64-token chunk and a partial one) equals 100 decode steps
    of the oracle: outputs, recurrent state and conv states."""
    B, T, H = 2, 100, 2
    a = _seq_inputs(B, T, H, 3, headwise)
    ref = {k: (v.clone() if k in ("csq", "csk", "csv", "state") else v) for k, v in a.items()}
    outs = []
    for t in range(T):
        step = {k: (v[:, t] if k in ("q", "k", "v", "g_proj", "beta", "g2") else v) for k, v in ref.items()}
        outs.append(KD.kda_decode_ref(**step))
    want = torch.stack(outs, 1).float()
    got = KD.kda_prefill(**a, chunk=64).float()
    assert got.shape == want.shape
    assert (got - want).abs().max().item() < 3e-2          # bf16 outputs: one rounding step apart at most
    assert torch.allclose(a["state"], ref["state"], rtol=1e-4, atol=1e-5)
    for c in ("csq", "csk", "csv"):
        assert torch.allclose(a[c], ref[c])


def test_small_projection_fuse_cpu():
    from inference_optimizations_b200.ops.kda import KDASmallProjections
    torch.manual_seed(0)
    H, nb, d, P, M = 256, 8, 32, 256, 37
    ws = [torch.randn(s, dtype=torch.bfloat16) * 0.05 for s in ((nb, H), (d, H), (P, d), (d, H), (P, d))]
    sp = KDASmallProjections(*ws)
    x = torch.randn(M, H, dtype=torch.bfloat16)
    ref = sp.forward_separate(x)
    sp.fuse()
    assert sp.w_a.shape == (nb + 2 * d, H) and sp.w_lr.shape == (2, d, P)
    assert sp.w_b.data_ptr() == sp.w_a.data_ptr()                  # separate weights now view the packed storage
    out = sp.forward(x)
    sep = sp.forward_separate(x)                                   # the separate path stays valid after the fuse
    for a, b, c in zip(ref, out, sep):
        assert a.shape == b.shape
        assert torch.allclose(a.float(), b.float(), atol=1e-2, rtol=1e-2)
        assert torch.equal(a, c)
