"""kvmix as the MLA serving pool on the GPU (FP8 block-scaled tiny DSA-MoE model, CUDA-graph decode): the writer kernel
sends each token's latent row to its request's pool, the sparse-MLA decode runs one launch per pool format (tokens of
the other pool skipped), so every request generates what a plain engine of its format generates; a promoted request's
rows are re-quantized into NVFP4 pages on the device."""
import pytest

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

pytestmark = pytest.mark.gpu

SHORT = [[(7 * i + 3 * j) % 500 + 1 for j in range(30 + 7 * i)] for i in range(2)]
LONG = [[(11 * i + 5 * j) % 500 + 1 for j in range(150 + 20 * i)] for i in range(2)]
PARAMS = SamplingParams(max_new_tokens=8)


def _engine(cuda, kv: str, **over) -> Engine:
    cfg = model_config("tiny_mla", expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8")
    ecfg = EngineConfig(model="tiny_mla", device=str(cuda), kv_dtype=kv, max_running=4, chunked_prefill=64,
                        graph_batch_sizes="1,2,4", prefix_cache=False, max_total_tokens=8192, **over)
    return Engine(ecfg, cfg, max_seq=512)


def test_kvmix_pool_matches_plain_pools_gpu(cuda):
    prompts = SHORT + LONG
    ref8 = _engine(cuda, "fp8").generate(prompts, PARAMS)
    ref4 = _engine(cuda, "nvfp4").generate(prompts, PARAMS)
    eng = _engine(cuda, "kvmix", kvmix_threshold=150)
    outs = eng.generate(prompts, PARAMS)
    assert outs[:2] == ref8[:2] and outs[2:] == ref4[2:], (outs, ref8, ref4)
    assert 4 in eng.runner.graphs and eng.runner.kv.alloc.used == 0
    eng.runner.kv.check()


def test_kvmix_promotion_gpu(cuda):
    eng = _engine(cuda, "kvmix", kvmix_threshold=10 ** 6)
    r = eng.add_request(SHORT[0], PARAMS)
    eng.step()
    assert eng.runner.pages[r.rid].fmt == "fp8"
    eng.runner.kv.alloc.mix.threshold = 33
    while eng.has_work():
        eng.step()
    assert eng.runner.promotions == 1 and len(r.output) == 8 and eng.runner.kv.alloc.used == 0
    eng.runner.kv.check()
