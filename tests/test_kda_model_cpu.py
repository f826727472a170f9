"""Hybrid Kimi-delta-attention + MLA + MoE family (`tiny_kda`: two KDA layers, one MLA layer) on CPU: the engine's
chunked prefill + decode (recurrent states carried per request row across chunks and steps) generates the greedy
continuation of a teacher-forced full-sequence pass; the recurrent state of a request row starts from zero."""
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams


def _engine(chunk: int = 24) -> Engine:
    ecfg = EngineConfig(model="tiny_kda", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=chunk,
                        cuda_graphs=False, prefix_cache=False)
    return Engine(ecfg, model_config("tiny_kda"), max_seq=256)


def test_kda_layers_and_states():
    eng = _engine()
    m = eng.runner.model
    assert [l.kda is not None for l in m.layers] == [True, True, False]
    assert sorted(eng.runner.kv.kda) == [0, 1]


def test_kda_hybrid_generation_matches_full_recompute():
    torch.manual_seed(3)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (50, 13, 77)]
    eng = _engine()
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=5))
    ref = _engine(chunk=512)                     # one prefill chunk per sequence, no decode steps
    for p, o in zip(prompts, outs):
        seq = list(p)
        for tok in o:
            logits = ref.runner.score(seq)[-1]
            top2 = torch.topk(logits, 2).values
            if (top2[0] - top2[1]).item() > 1e-2:
                assert tok == int(logits.argmax()), (len(seq), tok, int(logits.argmax()))
            seq.append(tok)
    assert eng.runner.kv.alloc.used == 0
