"""MLA + DSA + MoE family on the GPU: router kernel == oracle; the tiny model's forward through the kernels stays
close to the same forward on the fp32 CPU oracles; the engine generates end to end."""
import pytest
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams
from inference_optimizations_b200.ops import moe as MOE

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("e,k,g,kg", [(256, 8, 8, 4), (8, 2, 2, 1), (160, 8, 1, 1), (64, 6, 4, 2)])
def test_router_kernel_matches_oracle(cuda, e, k, g, kg):
    torch.manual_seed(e)
    logits = torch.randn(37, e) * 2
    bias = torch.randn(e) * 0.1
    ids, w = MOE.route(logits.to(cuda), bias.to(cuda), k, g, kg, 2.5)
    rid, rw = MOE.route_ref(logits, bias, k, g, kg, 2.5)
    # same expert set (order may differ only on exact ties, absent with random logits)
    assert torch.equal(ids.cpu().sort(-1).values, rid.sort(-1).values)
    assert torch.allclose(w.cpu().sort(-1).values, rw.sort(-1).values, rtol=1e-4, atol=1e-5)


def _engine(device, kv="nvfp4"):
    ecfg = EngineConfig(model="tiny_mla", device=device, kv_dtype=kv, max_running=4, chunked_prefill=32,
                        cuda_graphs=False)
    return Engine(ecfg, model_config("tiny_mla"), max_seq=256)


@pytest.mark.parametrize("kv", ["nvfp4", "fp8"])
def test_mla_model_gpu_vs_cpu_oracles(cuda, kv):
    """Same weights on both devices: prefill logits through the kernels (E4M3 sparse attention, indexer, router) stay
    close to the fp32-oracle forward, and the engine generates end to end on the GPU."""
    from inference_optimizations_b200.engine.scheduler import Request, Segment
    torch.manual_seed(3)
    cfg = model_config("tiny_mla")
    gpu, cpu = _engine(str(cuda), kv), _engine("cpu", kv)
    cpu.runner.model.copy_from(gpu.runner.model)
    prompt = torch.randint(0, cfg.vocab, (90,)).tolist()
    logits = []
    for eng in (gpu, cpu):
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        x = eng.runner.model.forward(st, eng.runner.kv)
        logits.append(eng.runner.model.logits(x).float().cpu())
    cos = torch.nn.functional.cosine_similarity(logits[0], logits[1], dim=-1)
    assert cos.mean().item() > 0.98 and cos.min().item() > 0.9, (cos.mean().item(), cos.min().item())
    out = gpu.generate([prompt[:40], prompt[:7]], SamplingParams(max_new_tokens=6))
    assert all(len(o) == 6 for o in out)


@pytest.mark.parametrize("dn,dv,hi,efmt", [(128, 128, 64, "fp8"), (192, 256, 32, "nvfp4")])
def test_fused_glue_head_geometries_vs_cpu_oracle(cuda, dn, dv, hi, efmt):
    """The fused attention glue (`mla_prep_kv` / `mla_prep_q`, the FP8 a / b / o projections, the head-batched W_UK
    and W_UV products, the indexer) at the DeepSeek-V3.2 head geometry (q_nope 128, v 128, 64 indexer heads) and the
    GLM-5 one (q_nope 192, v 256, 32 indexer heads, NVFP4 experts): prefill logits stay close to the fp32-oracle
    forward of the same weights on the CPU, and decode steps run end to end."""
    from inference_optimizations_b200.engine.scheduler import Request, Segment
    over = dict(hidden=256, num_heads=8, q_lora=256, qk_nope=dn, v_head=dv, index_heads=hi, weight_dtype="fp8",
                expert_dtype=efmt, expert_ffn=256, dense_ffn=512)
    cfg = model_config("tiny_mla", **over)
    engines = []
    for dev in (str(cuda), "cpu"):
        ecfg = EngineConfig(model="tiny_mla", device=dev, kv_dtype="nvfp4", max_running=4, chunked_prefill=128,
                            cuda_graphs=False, prefix_cache=False)
        engines.append(Engine(ecfg, cfg, max_seq=256))
    gpu, cpu = engines
    mg = gpu.runner.model
    assert all(mg._fused_glue(mg.layers[i]) for i in range(cfg.num_layers))
    cpu.runner.model.copy_from(mg)
    torch.manual_seed(5)
    prompt = torch.randint(0, cfg.vocab, (90,)).tolist()
    logits = []
    for eng in (gpu, cpu):
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        x = eng.runner.model.forward(st, eng.runner.kv)
        logits.append(eng.runner.model.logits(x).float().cpu())
        eng.runner.detach(r)
    cos = torch.nn.functional.cosine_similarity(logits[0], logits[1], dim=-1)
    assert cos.mean().item() > 0.98 and cos.min().item() > 0.9, (cos.mean().item(), cos.min().item())
    out = gpu.generate([prompt[:70], prompt[:9]], SamplingParams(max_new_tokens=5))
    assert all(len(o) == 5 for o in out)
    for d in (gpu.runner.kv.idx_ws, gpu.runner.kv.mla_ws):
        assert all(int(ws.status.item()) == 0 for ws in d.values())


@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
def test_block_scaled_experts_in_model(cuda, fmt):
    """The MLA model with FP8 / NVFP4 block-scaled experts (grouped tcgen05 GEMMs) tracks its bf16 twin."""
    import torch.nn.functional as Fn
    from inference_optimizations_b200.models.mla import MLAModel
    from inference_optimizations_b200.ops import moe as MOE
    over = dict(expert_ffn=256, dense_ffn=512, weight_dtype=fmt, expert_dtype=fmt)
    cq = model_config("tiny_mla", **over)
    cb = model_config("tiny_mla", **dict(over, weight_dtype="bf16", expert_dtype="bf16"))
    mq, mb = MLAModel(cq, cuda, seed=3), MLAModel(cb, cuda, seed=3)
    mb.copy_from(mq)
    torch.manual_seed(0)
    x = (torch.randn(9, cq.hidden, device=cuda) * 0.5).to(torch.bfloat16)
    for i in range(cq.num_layers):
        yq, yb = mq._ffn(i, x), mb._ffn(i, x)
        cos = Fn.cosine_similarity(yq.float().flatten(), yb.float().flatten(), dim=0).item()
        assert cos > (0.99 if fmt == "fp8" else 0.95), (i, cos)


def test_mla_decode_cuda_graph_matches_eager(cuda):
    """Decode steps replayed from the per-bucket CUDA graph (FP8 block-scaled experts, padded bucket) produce the
    same greedy tokens as the eager path."""
    over = dict(expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8")
    cfg = model_config("tiny_mla", **over)
    outs = []
    for graphs in (False, True):
        ecfg = EngineConfig(model="tiny_mla", device=str(cuda), kv_dtype="nvfp4", max_running=4, chunked_prefill=64,
                            cuda_graphs=graphs, graph_batch_sizes="4", prefix_cache=False)
        eng = Engine(ecfg, cfg, max_seq=256)
        torch.manual_seed(11)
        prompts = [torch.randint(1, cfg.vocab, (n,)).tolist() for n in (70, 33, 5)]
        outs.append(eng.generate(prompts, SamplingParams(max_new_tokens=8)))
        if graphs:
            assert 4 in eng.runner.graphs
    assert outs[0] == outs[1], outs


def test_mla_mtp_speculation_gpu(cuda):
    """MTP speculation through the GPU kernels (FP8 block-scaled experts, NVFP4 latent rows) emits the plain greedy
    tokens."""
    over = dict(expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8")
    cfg = model_config("tiny_mla", **over)
    torch.manual_seed(4)
    prompts = [torch.randint(1, cfg.vocab, (n,)).tolist() for n in (66, 12)]
    outs = []
    for spec in (False, True):
        ecfg = EngineConfig(model="tiny_mla", device=str(cuda), kv_dtype="nvfp4", max_running=4, chunked_prefill=64,
                            cuda_graphs=False, spec=spec, spec_policy="always", prefix_cache=False)
        eng = Engine(ecfg, cfg, max_seq=256)
        outs.append(eng.generate(prompts, SamplingParams(max_new_tokens=8)))
    assert outs[0] == outs[1], outs


@pytest.mark.parametrize("e,k,g,kg,ks", [(256, 8, 8, 4, 3), (160, 8, 1, 1, 2), (256, 8, 8, 4, 1)])
def test_router_sums_split_k_partials(cuda, e, k, g, kg, ks):
    """The router kernel fed the router GEMM's split-K partials (summed in split order inside) picks the same
    experts with the same weights as the kernel fed the summed logits, and agrees with the oracle."""
    torch.manual_seed(e + ks)
    T = 21
    part = torch.randn(ks * T, e) * 1.5
    bias = torch.randn(e) * 0.1
    summed = part[:T].clone()
    for j in range(1, ks):
        summed += part[j * T:(j + 1) * T]
    ids, w = MOE.route(part.to(cuda), bias.to(cuda), k, g, kg, 2.5, ksplit=ks)
    ids1, w1 = MOE.route(summed.to(cuda), bias.to(cuda), k, g, kg, 2.5)
    assert torch.equal(ids, ids1) and torch.equal(w, w1)
    rid, rw = MOE.route_ref(summed, bias, k, g, kg, 2.5)
    assert torch.equal(ids.cpu().sort(-1).values, rid.sort(-1).values)
    assert torch.allclose(w.cpu().sort(-1).values, rw.sort(-1).values, rtol=1e-4, atol=1e-5)


def test_bf16_reference_pool_on_gpu(cuda):
    """The unquantized bf16 latent pool (the accuracy reference) on the GPU: the engine writes 1152-byte rows and
    attends in fp32 through torch; its prefill logits match the same engine on the CPU, and the FP8-weight model's
    NVFP4-pool engine stays close to it."""
    from inference_optimizations_b200.engine.scheduler import Request, Segment
    over = dict(hidden=256, num_heads=8, q_lora=256, qk_nope=128, v_head=128, index_heads=64, weight_dtype="fp8",
                expert_dtype="fp8", expert_ffn=256, dense_ffn=512)
    cfg = model_config("tiny_mla", **over)
    engs = {}
    for name, dev, kv in (("gpu_bf16", str(cuda), "bf16"), ("cpu_bf16", "cpu", "bf16"), ("gpu_nvfp4", str(cuda), "nvfp4")):
        ecfg = EngineConfig(model="tiny_mla", device=dev, kv_dtype=kv, max_running=2, chunked_prefill=128,
                            prefix_cache=False)
        engs[name] = Engine(ecfg, cfg, max_seq=256)
    src = engs["gpu_bf16"].runner.model
    assert engs["gpu_bf16"].runner.kv.latent[0].shape[1] == 1152 and not src.fuse_glue
    engs["cpu_bf16"].runner.model.copy_from(src)
    engs["gpu_nvfp4"].runner.model.copy_from(src)
    torch.manual_seed(8)
    prompt = torch.randint(0, cfg.vocab, (80,)).tolist()
    logits = {}
    for name, eng in engs.items():
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        logits[name] = eng.runner.model.logits(eng.runner.model.forward(st, eng.runner.kv)).float().cpu()
        eng.runner.detach(r)
    cos = lambda a, b: torch.nn.functional.cosine_similarity(logits[a], logits[b], dim=-1)  # noqa: E731
    assert cos("gpu_bf16", "cpu_bf16").min().item() > 0.98
    assert cos("gpu_nvfp4", "gpu_bf16").mean().item() > 0.95
    out = engs["gpu_bf16"].generate([prompt[:50]], SamplingParams(max_new_tokens=4))
    assert len(out[0]) == 4
