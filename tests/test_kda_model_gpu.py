"""Hybrid Kimi-delta-attention + MLA + MoE family on the GPU (FP8 block-scaled MLA projections and experts, bf16 KDA
projections on the framework's GEMM, the fused KDA decode kernel with per-request states gathered / scattered by row):
CUDA-graph decode equals eager decode, and generation follows a teacher-forced full-sequence pass (chunked prefill
through torch ops vs the decode kernel: equal up to rounding, so near-ties may differ)."""
import pytest
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

pytestmark = pytest.mark.gpu


def _engine(cuda, graphs: bool, chunk: int = 64) -> Engine:
    cfg = model_config("tiny_kda", expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8")
    ecfg = EngineConfig(model="tiny_kda", device=str(cuda), kv_dtype="nvfp4", max_running=4, chunked_prefill=chunk,
                        cuda_graphs=graphs, graph_batch_sizes="4", prefix_cache=False)
    return Engine(ecfg, cfg, max_seq=512)


def test_kda_hybrid_graph_equals_eager_and_follows_recompute(cuda):
    torch.manual_seed(8)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (90, 21, 140)]
    params = SamplingParams(max_new_tokens=8)
    eager = _engine(cuda, False).generate(prompts, params)
    eng = _engine(cuda, True)
    graph = eng.generate(prompts, params)
    assert 4 in eng.runner.graphs and graph == eager, (graph, eager)
    ref = _engine(cuda, False, chunk=512)
    agree, total = 0, 0
    for p, o in zip(prompts, graph):
        seq = list(p)
        for tok in o:
            agree += int(tok == int(ref.runner.score(seq)[-1].argmax()))
            total += 1
            seq.append(tok)
    assert agree / total >= 0.9, (agree, total)
