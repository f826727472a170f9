"""Engine on the GPU kernel path: paged prefill + CUDA-graph decode against the cache-free reference."""
import pytest
import torch

from inference_optimizations_b200.config import EngineConfig
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("graphs", [False, True])
def test_engine_matches_reference_bf16_kv(cuda, graphs):
    torch.manual_seed(0)
    ecfg = EngineConfig(model="tiny_gqa", device="cuda:0", kv_dtype="bf16", max_running=4, chunked_prefill=64,
                        cuda_graphs=graphs, graph_batch_sizes="1,2,4")
    eng = Engine(ecfg, max_seq=512)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (130, 17, 77)]
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=6))
    checked = 0
    for p, o in zip(prompts, outs):
        seq = list(p)
        for tok in o:
            ref = eng.runner.model.reference_logits(seq)[-1]
            top2 = torch.topk(ref, 2).values
            if (top2[0] - top2[1]).item() > 0.05:
                assert tok == int(ref.argmax())
                checked += 1
            seq.append(tok)
    assert checked >= 8


@pytest.mark.parametrize("kv", ["nvfp4", "fp8"])
def test_engine_quantized_kv_runs(cuda, kv):
    ecfg = EngineConfig(model="tiny_gqa", device="cuda:0", kv_dtype=kv, max_running=4, chunked_prefill=64,
                        graph_batch_sizes="1,2,4")
    eng = Engine(ecfg, max_seq=512)
    prompts = [[(i * 13 + j) % 500 + 1 for j in range(30 + 40 * i)] for i in range(4)]
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=5))
    assert all(len(o) == 5 for o in outs)
    assert eng.runner.kv.alloc["global"].used == 0


def test_speculative_decoding_gpu_matches_reference(cuda):
    torch.manual_seed(3)
    ecfg = EngineConfig(model="tiny_gqa", device="cuda:0", kv_dtype="bf16", max_running=4, chunked_prefill=64,
                        graph_batch_sizes="1,2,4", spec=True, draft_tokens=3)
    eng = Engine(ecfg, max_seq=512)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (90, 41, 150)]
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=10))
    checked = 0
    for p, o in zip(prompts, outs):
        seq = list(p)
        for tok in o:
            ref = eng.runner.model.reference_logits(seq)[-1]
            top2 = torch.topk(ref, 2).values
            if (top2[0] - top2[1]).item() <= 0.05:
                break
            assert tok == int(ref.argmax())
            checked += 1
            seq.append(tok)
    assert checked >= 6
    assert all(r.spec_steps > 0 for r in eng.finished)
