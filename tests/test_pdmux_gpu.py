"""SM-partitioned prefill / decode lanes on a B200: green-context partitions confine work to their SMs, and the lanes
generate exactly the plain engine's tokens (same kernels; the prefill advances a few layers per iteration on its own
partition while CUDA-graph decode steps run on the other)."""
import pytest
import torch

from inference_optimizations_b200.config import EngineConfig
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.pdmux import Lanes, PdmuxEngine
from inference_optimizations_b200.engine.scheduler import SamplingParams

pytestmark = pytest.mark.gpu

PROMPTS = [list(range(3, 160)), list(range(7, 16)), list(range(100, 390)), list(range(1, 33))]


def _ms(fn, stream, n=10):
    with torch.cuda.stream(stream):
        fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / n


def test_sm_lanes_partition():
    lanes = Lanes("cuda:0", 3)
    p, d = lanes.streams(1)
    p_sms, d_sms = lanes.sms[1]
    total = torch.cuda.get_device_properties(0).multi_processor_count
    assert p_sms > 0 and d_sms > 0 and p_sms + d_sms <= total and d_sms % 8 == 0
    a = torch.randn(8192, 8192, device="cuda", dtype=torch.bfloat16)
    ref = a @ a
    full = _ms(lambda: a @ a, torch.cuda.Stream())
    part = _ms(lambda: a @ a, p)
    with torch.cuda.stream(d):
        b = a @ a
    torch.cuda.synchronize()
    assert torch.equal(b, ref)
    print(f"8192^3 bf16 GEMM: all SMs {full:.3f} ms, prefill lane ({p_sms} SMs) {part:.3f} ms")
    assert part > 1.3 * full          # the partition really holds fewer SMs


@pytest.mark.parametrize("kv", ["nvfp4", "bf16"])
def test_pdmux_matches_plain_engine(kv):
    params = SamplingParams(max_new_tokens=8, ignore_eos=True)
    ecfg = EngineConfig(model="tiny_gqa", device="cuda:0", kv_dtype=kv, max_running=4, chunked_prefill=128)
    ref = Engine(ecfg, max_seq=1024).generate(PROMPTS, params)
    pm = PdmuxEngine(Engine(ecfg, max_seq=1024), token_budget=256)     # 2 layers per iteration of a 128-token chunk
    outs = pm.generate(PROMPTS, params)
    assert outs == ref
    assert any(g == 1 and s is not None and n > 0 for g, s, n in pm.log)   # both lanes busy on the split partitions
    assert pm.engine.runner.kv.alloc["global"].used == 0


def test_pdmux_five_groups():
    """Five stream groups: the decode batch picks the largest decode partition; tokens stay the plain engine's."""
    params = SamplingParams(max_new_tokens=6, ignore_eos=True)
    ecfg = EngineConfig(model="tiny_gqa", device="cuda:0", kv_dtype="nvfp4", max_running=4, chunked_prefill=128)
    ref = Engine(ecfg, max_seq=1024).generate(PROMPTS, params)
    pm = PdmuxEngine(Engine(ecfg, max_seq=1024), n_groups=5, token_budget=256, decode_bs_divisor=1)
    assert pm.generate(PROMPTS, params) == ref
    used = {g for g, s, n in pm.log if s is not None and n > 0}
    assert used == {3}
    assert pm.lanes.sms[3][1] > pm.lanes.sms[3][0]


def test_pdmux_mla_family_matches_plain_engine():
    """The DSA-MoE family (FP8 block-scaled projections and experts, NVFP4 latent KV) through the lanes: prefill split
    by layer ranges on the prefill partition beside CUDA-graph decode on the decode partition gives the plain
    engine's tokens; the split's launches use their own scratch buffers (a chunk of a decode batch's size included)."""
    from inference_optimizations_b200.config import model_config
    cfg = model_config("tiny_mla", expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8")
    params = SamplingParams(max_new_tokens=8, ignore_eos=True)
    ecfg = EngineConfig(model="tiny_mla", device="cuda:0", kv_dtype="nvfp4", max_running=4, chunked_prefill=64,
                        graph_batch_sizes="1,2,4", prefix_cache=False)
    ref = Engine(ecfg, cfg, max_seq=1024).generate(PROMPTS, params)
    pm = PdmuxEngine(Engine(ecfg, cfg, max_seq=1024), token_budget=64)     # one layer per iteration of a chunk
    outs = pm.generate(PROMPTS, params)
    assert outs == ref
    assert any(g == 1 and s is not None and n > 0 for g, s, n in pm.log)
    assert pm.engine.runner.kv.alloc.used == 0
