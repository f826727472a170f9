"""Operator tooling on CPU: accuracy gate metrics and engine scoring."""
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.tooling import accuracy_gate as G


def _eng(kv, model="tiny_gqa"):
    return Engine(EngineConfig(model=model, device="cpu", kv_dtype=kv, max_running=2, chunked_prefill=64,
                               cuda_graphs=False), model_config(model), max_seq=128)


def test_gate_metrics_identity_and_shift():
    ref = torch.randn(10, 50)
    c = G.compare_logits(ref, ref)
    assert c["kl"].abs().max() < 1e-6 and c["top1"].min() == 1
    c = G.compare_logits(ref, ref + 1.0)             # a constant shift leaves the distribution unchanged
    assert c["kl"].abs().max() < 1e-5


def test_gate_nvfp4_vs_bf16_kv_on_tiny_models():
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 512, (60,), generator=g).tolist() for _ in range(3)]
    same = G.run_gate(_eng("bf16"), _eng("bf16"), prompts)
    assert same.kl_mean < 1e-6 and same.top1 == 1.0
    q = G.run_gate(_eng("bf16"), _eng("nvfp4"), prompts)
    assert 0 < q.kl_mean < 0.5 and q.positions == 3 * 59
    m = G.run_gate(_eng("fp8", "tiny_mla"), _eng("nvfp4", "tiny_mla"), prompts)
    assert m.kl_mean >= 0 and m.positions == 3 * 59


def test_safetensors_roundtrip_and_tp_sharding(tmp_path):
    from inference_optimizations_b200.models import loader as L
    from inference_optimizations_b200.models.gqa import GQAModel
    cfg = model_config("tiny_gqa")
    full = GQAModel(cfg, "cpu", seed=3)
    path = str(tmp_path / "m.safetensors")
    L.export_gqa(full, path)
    idx = L.open_checkpoint(path)
    # tp=1 round trip is exact
    m1 = GQAModel(cfg, "cpu", weights=L.shard_gqa(idx, cfg, 0, 1, "cpu"))
    for a, b in zip(full.layers, m1.layers):
        assert torch.equal(a.qkv, b.qkv) and torch.equal(a.o, b.o) and torch.equal(a.down, b.down)
    # tp=2 shards reassemble the checkpoint; random init with tp=2 gives the same shards (TP-invariant init)
    for r in range(2):
        sh = L.shard_gqa(idx, cfg, r, 2, "cpu")
        mr = GQAModel(cfg, "cpu", r, 2, seed=3)
        assert torch.equal(sh["model.layers.0.self_attn.o_proj.weight"], mr.layers[0].o)
        assert torch.equal(sh["model.embed_tokens.weight"], mr.embed)


def test_bounds_check_catches_bad_page_table():
    import pytest
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    from inference_optimizations_b200.tooling.bounds import BoundsError
    for model in ("tiny_gqa", "tiny_mla"):
        ecfg = EngineConfig(model=model, device="cpu", kv_dtype="nvfp4", max_running=2, chunked_prefill=32,
                            cuda_graphs=False, bounds_check=True)
        eng = Engine(ecfg, model_config(model), max_seq=128)
        eng.generate([[1, 2, 3] * 5], SamplingParams(max_new_tokens=2))          # clean run passes the checks
        r = eng.add_request([4, 5, 6] * 5, SamplingParams(max_new_tokens=4))
        eng.step()                                                               # prefill
        table = eng.runner.kv.tables["global"] if model == "tiny_gqa" else eng.runner.kv.table
        table.host[r.slot, 0] = 10 ** 6                                           # corrupt: not a page
        table._dirty.add(r.slot)
        with pytest.raises(BoundsError):
            eng.step()


def test_serving_gate_ab_record():
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.tooling import serving_gate as SG
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="nvfp4", max_running=3, chunked_prefill=64,
                        cuda_graphs=False)
    res = SG.gate(ecfg, model_config("tiny_gqa"), {"decode_burst": 2}, sessions=3, prompt=40, steps=3, warmup=1,
                  repeats=2)
    assert set(res["arms"]) == {"control", "delta"}
    for arm in res["arms"].values():
        assert len(arm["runs"]) == 2 and all(r["tokens"] > 0 for r in arm["runs"])
        assert arm["config_digest"]
    assert res["arms"]["control"]["config_digest"] != res["arms"]["delta"]["config_digest"]
    assert res["verdict"] in ("neutral", "better", "worse")
