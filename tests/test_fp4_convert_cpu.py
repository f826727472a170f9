"""INT4 -> NVFP4 / MXFP4 conversion (tooling/fp4_convert.py): INT4 pack round trip, exactness when the INT4 grid
fits E2M1, the scale-window search never losing to the nominal scale (block by block), only storable scales written,
and a streamed checkpoint conversion with its report."""
import json
import os

import torch

from inference_optimizations_b200.tooling import fp4_convert as C


def _int4(out, cols, seed):
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(-8, 8, (out, cols), generator=g, dtype=torch.int8)
    scale = (torch.rand(out, cols // 32, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    return codes, scale


def test_int4_pack_round_trip():
    codes, _ = _int4(5, 96, 0)
    assert torch.equal(C.unpack_int4(C.pack_int4(codes), 96), codes)


def test_e2m1_subset_grid_is_exact():
    # codes in {0, +-1, +-2, +-3, +-4, +-6} times one scale per block are exactly representable in NVFP4
    g = torch.Generator().manual_seed(1)
    allowed = torch.tensor([0, 1, 2, 3, 4, 6, -1, -2, -3, -4, -6], dtype=torch.float32)
    w = allowed[torch.randint(0, 11, (8, 64), generator=g)] * 0.5
    w[:, ::16] = 6.0 * 0.5                          # amax fixes the scale at 0.5 exactly
    q, s8, g2 = C.quant_nvfp4(w, search=True, global_scale=1.0)
    assert torch.equal(C.dequant_nvfp4(q, s8, g2), w)


def test_search_not_worse_than_plain():
    codes, scale = _int4(64, 256, 2)
    ref = codes.float() * scale.float().repeat_interleave(32, 1)
    for quant, deq, blk in ((C.quant_nvfp4, lambda t: C.dequant_nvfp4(*t), 16),
                            (C.quant_mxfp4, lambda t: C.dequant_mxfp4(*t), 32)):
        ds, dp = deq(quant(ref, True)), deq(quant(ref, False))
        es = ((ds - ref) ** 2).view(64, -1, blk).sum(-1)
        ep = ((dp - ref) ** 2).view(64, -1, blk).sum(-1)
        assert (es <= ep * (1 + 1e-6) + 1e-12).all()              # per block: the nominal scale is a candidate
        rs, rp = C.report(ref, ds), C.report(ref, dp)
        assert rs["sqnr_db"] >= rp["sqnr_db"] - 1e-6 and rs["sqnr_db"] > 18, (rs, rp)


def test_nvfp4_scales_are_storable_and_global_is_modelopt():
    codes, scale = _int4(16, 128, 3)
    ref = codes.float() * scale.float().repeat_interleave(32, 1)
    q, s8, g2 = C.quant_nvfp4(ref)
    assert s8.dtype == torch.float8_e4m3fn and torch.isfinite(s8.float()).all() and (s8.float() > 0).all()
    want = float(ref.abs().max()) / (6 * 448)
    assert abs(float(g2) - want) < 1e-6 * want                   # fp32-stored global scale
    assert torch.allclose(C.dequant_nvfp4(q, s8, g2).abs().max(), ref.abs().max(), rtol=0.2)


def test_streamed_checkpoint_conversion(tmp_path):
    from inference_optimizations_b200.models.loader import SafeTensors, save
    src, dst = tmp_path / "src", tmp_path / "dst"
    os.makedirs(src)
    for shard in range(2):
        t = {}
        for e in range(2):
            codes, scale = _int4(128, 256, 10 * shard + e)
            p = f"model.layers.{shard}.mlp.experts.{e}.down_proj"
            t[p + ".weight_packed"] = C.pack_int4(codes)
            t[p + ".weight_scale"] = scale
            t[p + ".weight_shape"] = torch.tensor([128, 256], dtype=torch.int32)
        t[f"model.layers.{shard}.input_layernorm.weight"] = torch.ones(256, dtype=torch.bfloat16)
        save(t, str(src / f"model-{shard:05d}.safetensors"))
    stats = C.convert(str(src), str(dst), "nvfp4")
    assert len(stats) == 4 and min(v["sqnr_db"] for v in stats.values()) > 18
    st = SafeTensors(str(dst / "model-00001.safetensors"))
    keys = set(st.keys())
    assert "model.layers.1.mlp.experts.0.down_proj.weight" in keys
    assert "model.layers.1.mlp.experts.0.down_proj.weight_scale_2" in keys
    assert "model.layers.1.input_layernorm.weight" in keys
    assert st.get("model.layers.1.mlp.experts.0.down_proj.weight").shape == (128, 128)
    assert json.load(open(dst / "conversion_report.json"))["format"] == "nvfp4"
