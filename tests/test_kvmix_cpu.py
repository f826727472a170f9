"""kvmix (kv/kvmix.py): one page-id space over FP8 and NVFP4 MLA pools, length-based placement, cross-pool fallback,
promotion FP8 -> NVFP4 equal to quantizing the FP8-dequantized latents directly, capacity accounting."""
import pytest
import torch

from inference_optimizations_b200.kv import kvmix as KM
from inference_optimizations_b200.ops import formats as F


def test_page_space_and_fallback():
    a = KM.KVMixAllocator(pages_fp8=4, pages_fp4=6, threshold=1000)
    assert a.preferred(999) == "fp8" and a.preferred(1000) == "nvfp4"
    p8 = a.alloc(3, "fp8")
    assert all(not a.is_fp4(p) for p in p8) and sorted(a.local(p) for p in p8) == [0, 1, 2]
    p = a.alloc(2, "fp8")                          # only one FP8 page left: served from FP4
    assert all(a.is_fp4(x) for x in p) and a.fallbacks == 1
    with pytest.raises(KM.PoolExhausted):
        a.alloc(9, "nvfp4")
    a.release(p8 + p)
    assert a.free_tokens == 64 * 10


def test_promotion_requantizes_rows_and_frees_fp8_pages():
    torch.manual_seed(0)
    a = KM.KVMixAllocator(pages_fp8=8, pages_fp4=8, threshold=150)
    layers = [KM.KVMixPools(a, "cpu") for _ in range(2)]
    req = KM.KVMixRequest(a, total_len_hint=100)
    assert req.fmt == "fp8"
    n = 140
    req.ensure(n, layers)
    lat = [torch.randn(n, 576) for _ in layers]
    for L, x in zip(layers, lat):
        L.write(x[:, :512], x[:, 512:], req.pages, torch.arange(n))
    free8 = len(a.free8)
    fp8_vals = [F.mla_fp8_row_dequantize(torch.cat([L.fp8[a.local(p) * 64:a.local(p) * 64 + 64] for p in req.pages])[:n])
                for L in layers]
    assert req.ensure(160, layers) is True          # crossing the threshold promotes every layer
    assert req.fmt == "nvfp4" and all(a.is_fp4(p) for p in req.pages)
    assert len(a.free8) == free8 + 3                # the three FP8 pages came back
    for L, v in zip(layers, fp8_vals):
        rows = torch.cat([L.fp4[a.local(p) * 64:a.local(p) * 64 + 64] for p in req.pages])[:n]
        want = F.mla_row_quantize(v[:, :512], v[:, 512:])
        assert torch.equal(rows, want)
    req.free()
    assert a.free_tokens == 64 * 16


def test_capacity_gain():
    assert abs(KM.capacity_gain(576 * 1000, 1.0) - 576 / 352) < 1e-9
    assert KM.capacity_gain(576 * 1000, 0.0) == 1.0
