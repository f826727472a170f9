"""Rope-free 288-byte NVFP4 rows and DeepSeek V4 Pro 320/384-byte cells (ops/formats.py): layout, exact round trip
on the FP4 grid, error bound, the scale search never losing to the plain scale, ties-to-even rounding."""
import torch

from inference_optimizations_b200.ops import formats as F


def test_glmflash_row_is_the_mla_row_without_rope():
    torch.manual_seed(0)
    nope, rope = torch.randn(9, 512), torch.randn(9, 64)
    r288 = F.glmflash_row_quantize(nope)
    r352 = F.mla_row_quantize(nope, rope)
    assert r288.shape == (9, 288) and torch.equal(r288, r352[:, :288])
    d = F.glmflash_row_dequantize(r288)
    assert torch.equal(d, F.mla_row_dequantize(r352)[:, :512])


def test_v4pro_cell_layout_and_round_trip():
    torch.manual_seed(1)
    x = torch.randn(17, 512) * torch.exp2(torch.randint(-4, 5, (17, 1)).float())
    for rope, nbytes in (("fp8", 320), ("bf16", 384)):
        c = F.v4pro_cell_quantize(x, rope)
        assert c.shape == (17, nbytes)
        assert torch.all(c[:, 252:256] == 0)
        d = F.v4pro_cell_dequantize(c, rope)
        # values already on the grid survive exactly
        assert torch.equal(F.v4pro_cell_quantize(d, rope), c)
        err = (d[:, :448] - x[:, :448]).reshape(17, 28, 16)
        amax = x[:, :448].abs().reshape(17, 28, 16).amax(-1, keepdim=True)
        assert torch.all(err.abs() <= amax * (1 / 6 + 1 / 4) + 1e-6)
        if rope == "bf16":
            assert torch.equal(d[:, 448:], x[:, 448:].to(torch.bfloat16).float())


def test_v4pro_scale_search_beats_plain_scale():
    torch.manual_seed(2)
    x = torch.randn(64, 512)
    c = F.v4pro_cell_quantize(x)
    d = F.v4pro_cell_dequantize(c)
    # the plain rule alone (f = 1)
    saved = F.V4P_SCALE_SEARCH
    try:
        F.V4P_SCALE_SEARCH = (1.0,)
        d1 = F.v4pro_cell_dequantize(F.v4pro_cell_quantize(x))
    finally:
        F.V4P_SCALE_SEARCH = saved
    e_search = (d[:, :448] - x[:, :448]).pow(2).reshape(64, 28, 16).sum(-1)
    e_plain = (d1[:, :448] - x[:, :448]).pow(2).reshape(64, 28, 16).sum(-1)
    assert torch.all(e_search <= e_plain + 1e-12) and e_search.sum() < e_plain.sum()


def test_e2m1_ties_to_even():
    m = F._e2m1_mag_even(torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0]))
    assert m.tolist() == [0, 2, 2, 4, 4, 6, 6, 7]
