"""Row formats: bit-level rules of the NVFP4 MLA row, FP8 rows, indexer keys (CPU oracles)."""
import torch

from inference_optimizations_b200.ops import formats as F


def test_layout_constants():
    assert (F.MLA_SCALE_OFF, F.MLA_ROPE_OFF, F.MLA_ROW_BYTES) == (256, 288, 352)
    assert F.MLA_FP8_ROW_BYTES == 576 and F.INDEX_ROW_BYTES == 132


def test_nibble_order_and_grid_exact():
    # values exactly on the E2M1 grid times a power-of-two scale survive bit-exactly
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0] * 2)
    vals[8:] *= -1
    vals[8] = 0.0
    nope = torch.zeros(1, 512)
    nope[0, :16] = vals
    rows = F.mla_row_quantize(nope, torch.zeros(1, 64))
    # block 0 amax = 6 -> scale 1.0
    assert rows[0, 256].item() == torch.tensor(1.0).to(torch.float8_e4m3fn).view(torch.uint8).item()
    # element 0 (0.0) low nibble, element 1 (0.5) high nibble of byte 0
    assert rows[0, 0].item() == (0 | (1 << 4))
    back = F.mla_row_dequantize(rows)
    assert torch.equal(back[0, :16], vals)


def test_ties_round_down_and_saturate():
    y = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.25, -0.1, 0.2500001])
    codes = F.e2m1_encode(y)
    assert codes.tolist() == [0, 1, 2, 3, 4, 5, 6, 7, 0, 0, 1]  # no negative zero: -0.25 -> code 0


def test_roundtrip_error_bound():
    torch.manual_seed(0)
    nope = torch.randn(64, 512) * 3
    rope = torch.randn(64, 64)
    rows = F.mla_row_quantize(nope, rope)
    back = F.mla_row_dequantize(rows)
    blk = nope.reshape(64, 32, 16).abs().amax(-1, keepdim=True)
    err = (back[:, :512] - nope).reshape(64, 32, 16).abs()
    # half an E2M1 step at the top (1.0 of 6 -> amax/6) plus the E4M3 scale rounding (<= 1/16 relative)
    assert bool((err <= blk * (1 / 6 + 1 / 8) + 1e-6).all())
    assert torch.equal(back[:, 512:], rope.to(torch.float8_e4m3fn).float())


def test_scale_clamp_and_zero_rows():
    rows = F.mla_row_quantize(torch.zeros(2, 512), torch.zeros(2, 64))
    s = rows[:, 256:288].view(torch.float8_e4m3fn).float()
    assert torch.all(s == 2.0 ** -9)
    assert torch.all(F.mla_row_dequantize(rows) == 0)
    big = F.mla_row_quantize(torch.full((1, 512), 1e6), torch.zeros(1, 64))
    assert torch.all(big[:, 256:288].view(torch.float8_e4m3fn).float() == 448.0)


def test_fp8_row_and_index_key():
    torch.manual_seed(1)
    nope, rope = torch.randn(8, 512), torch.randn(8, 64)
    r = F.mla_fp8_row_quantize(nope, rope)
    assert r.shape == (8, 576)
    assert torch.allclose(F.mla_fp8_row_dequantize(r), torch.cat([nope, rope], -1), rtol=0.07, atol=0.02)
    k = torch.randn(8, 128)
    kr = F.index_key_quantize(k)
    assert kr.shape == (8, 132)
    assert torch.allclose(F.index_key_dequantize(kr), k, rtol=0.07, atol=0.03)


def test_nvfp4_generic_with_global_scale():
    torch.manual_seed(2)
    x = torch.randn(4, 3, 256) * 50
    p, s = F.nvfp4_quantize(x, global_scale=8.0)
    back = F.nvfp4_dequantize(p, s, 8.0)
    blk = x.reshape(4, 3, 16, 16).abs().amax(-1, keepdim=True)
    err = (back - x).reshape(4, 3, 16, 16).abs()
    assert bool((err <= blk * (1 / 6 + 1 / 8) + 1e-5).all())


def test_ue8m0_fp8_quant():
    torch.manual_seed(3)
    x = torch.randn(5, 256) * 10
    q, s = F.fp8_quant_ue8m0(x)
    assert torch.all(torch.log2(s) == torch.round(torch.log2(s)))
    back = (q.float().reshape(5, 2, 128) * s[..., None]).reshape(5, 256)
    assert torch.allclose(back, x, rtol=0.07, atol=1e-3)
