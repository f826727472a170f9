"""MLA-family checkpoints on CPU: a random-init model exported in the HuggingFace DeepSeek-V3 layout (bf16 and FP8
with 128x128 block scales, rope rows interleaved as the checkpoints store them) loads back into the same weights; an
expert-parallel rank reads only its experts; an engine pointed at the checkpoint generates what the original model
generates."""
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams
from inference_optimizations_b200.models import mla_loader as ML
from inference_optimizations_b200.models.mla import MLAModel

FIELDS = ("n_in", "n_post", "wq_a", "q_norm", "wq_b", "wkv_a", "kv_norm", "w_uk", "w_uv", "wo", "wi_q", "wi_k",
          "wi_kn", "wi_kb", "wi_w")


def _pairs(a, b):
    yield "embed", a.embed, b.embed
    yield "lm_head", a.lm_head, b.lm_head
    yield "final_norm", a.final_norm, b.final_norm
    for i, (la, lb) in enumerate(zip(a.layers, b.layers)):
        for f in FIELDS:
            yield f"{i}.{f}", getattr(la, f), getattr(lb, f)
        for k, v in la.ffn.items():
            if v is not None:
                yield f"{i}.ffn.{k}", v, lb.ffn[k]
    if a.draft:
        for f in ("eh_proj", "enorm", "hnorm", "draft_norm"):
            yield f, getattr(a, f), getattr(b, f)


def test_roundtrip_bf16(tmp_path):
    cfg = model_config("tiny_mla")
    a = MLAModel(cfg, "cpu", seed=5, keep_master=True)
    a.build_draft()
    files = ML.export_hf(a, str(tmp_path))
    assert files and (tmp_path / "config.json").exists()
    b = ML.load_mla(str(tmp_path), cfg, "cpu", keep_master=True, draft=True)
    n = 0
    for name, x, y in _pairs(a, b):
        assert torch.equal(x, y), name
        n += 1
    assert n > 50


def test_roundtrip_fp8_block_scaled(tmp_path):
    cfg = model_config("tiny_mla")
    a = MLAModel(cfg, "cpu", seed=6, keep_master=True)
    ML.export_hf(a, str(tmp_path), fp8=True)
    from inference_optimizations_b200.models.loader import open_checkpoint
    idx = open_checkpoint(str(tmp_path))
    assert idx["model.layers.0.self_attn.q_a_proj.weight"].get("model.layers.0.self_attn.q_a_proj.weight").dtype == \
        torch.float8_e4m3fn
    b = ML.load_mla(str(tmp_path), cfg, "cpu", keep_master=True)
    for name, x, y in _pairs(a, b):
        if x.dim() >= 2 and "gate" not in name.split(".")[-1] and name != "embed":
            q, s = ML.quant_fp8_blocks(x.float().reshape(-1, x.shape[-1]))
            want = ML.dequant_fp8_blocks(q, s).to(torch.bfloat16)
            err = (y.float() - x.float()).abs().max() / x.float().abs().max()
            assert err < 0.07, (name, float(err))
            if y.dim() == 2 and name.endswith(("wq_a", "wo", "wi_k", "wi_w")):
                assert torch.equal(y, want), name
        else:
            assert torch.equal(x, y), name


def test_ep_rank_reads_its_experts(tmp_path):
    cfg = model_config("tiny_mla")
    a = MLAModel(cfg, "cpu", seed=7, keep_master=True)
    ML.export_hf(a, str(tmp_path))
    b = ML.load_mla(str(tmp_path), cfg, "cpu", ep_rank=1, ep_world=2, keep_master=True)
    E = cfg.num_experts
    for i in range(cfg.num_layers):
        if cfg.is_moe(i):
            assert torch.equal(b.layers[i].ffn["w_gu"], a.layers[i].ffn["w_gu"][E // 2:])
            assert torch.equal(b.layers[i].ffn["w_down"], a.layers[i].ffn["w_down"][E // 2:])


def test_engine_serves_the_checkpoint(tmp_path):
    cfg = model_config("tiny_mla")
    a = MLAModel(cfg, "cpu", seed=11, keep_master=True)
    ML.export_hf(a, str(tmp_path))
    prompts = [[(5 * i + 3 * j) % 400 + 1 for j in range(70 + 20 * i)] for i in range(2)]
    mk = lambda **kw: Engine(EngineConfig(model="tiny_mla", device="cpu", kv_dtype="fp8", max_running=2,  # noqa: E731
                                          chunked_prefill=64, cuda_graphs=False, **kw), cfg, max_seq=256)
    ref = mk(seed=11).generate(prompts, SamplingParams(max_new_tokens=5))
    got = mk(seed=999, checkpoint=str(tmp_path)).generate(prompts, SamplingParams(max_new_tokens=5))
    assert got == ref
