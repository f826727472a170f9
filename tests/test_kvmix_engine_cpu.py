"""kvmix as the MLA serving pool (CPU, torch reference path): FP8 and NVFP4 latent rows in one page-id space, each
request placed in one pool by length with cross-pool fallback, promotion FP8 -> NVFP4 when a request grows past the
threshold.  Attention reads every token's rows from its request's pool, so a request's outputs equal those of a
plain engine holding the whole pool in that request's format."""
from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams

SHORT = [[(7 * i + 3 * j) % 500 + 1 for j in range(30 + 7 * i)] for i in range(2)]
LONG = [[(11 * i + 5 * j) % 500 + 1 for j in range(150 + 20 * i)] for i in range(2)]
PARAMS = SamplingParams(max_new_tokens=6)


def _engine(kv: str, **over) -> Engine:
    ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype=kv, max_running=4, chunked_prefill=64,
                        cuda_graphs=False, prefix_cache=False, max_total_tokens=4096, **over)
    return Engine(ecfg, model_config("tiny_mla"), max_seq=256)


def test_placement_by_length_matches_plain_pools():
    """Threshold 150: the short prompts live in FP8 pages, the long ones in NVFP4 pages; each request generates what
    the plain FP8 / NVFP4 engine generates for it."""
    prompts = SHORT + LONG
    ref8 = _engine("fp8").generate(prompts, PARAMS)
    ref4 = _engine("nvfp4").generate(prompts, PARAMS)
    eng = _engine("kvmix", kvmix_threshold=150)
    reqs = [eng.add_request(p, PARAMS) for p in prompts]
    fmts = {}
    while eng.has_work():
        eng.step()
        for r in reqs:
            rp = eng.runner.pages.get(r.rid)
            if rp is not None:
                fmts[r.rid] = rp.fmt
    assert [fmts[r.rid] for r in reqs] == ["fp8", "fp8", "nvfp4", "nvfp4"]
    outs = [r.output for r in reqs]
    assert outs[:2] == ref8[:2] and outs[2:] == ref4[2:], (outs, ref8, ref4)
    assert eng.runner.kv.alloc.used == 0


def test_fallback_and_promotion():
    """A tiny FP8 share sends requests that prefer FP8 to the NVFP4 pool (fallback); a request that grows past the
    threshold while decoding is promoted: its rows re-quantized into NVFP4 pages, its FP8 pages freed."""
    eng = _engine("kvmix", kvmix_threshold=10 ** 6, kvmix_fp8_share=0.02)
    out = eng.generate(SHORT, PARAMS)
    assert all(len(o) == 6 for o in out) and eng.runner.kv.alloc.mix.fallbacks >= 1
    eng = _engine("kvmix", kvmix_threshold=10 ** 6)
    reqs = [eng.add_request(SHORT[0], PARAMS)]          # placed in FP8 at admission
    eng.step()                                           # prefill: 30 tokens in FP8 pages
    assert eng.runner.pages[reqs[0].rid].fmt == "fp8"
    eng.runner.kv.alloc.mix.threshold = 33              # the request will cross it on its third decode step
    seen = set()
    while eng.has_work():
        eng.step()
        rp = eng.runner.pages.get(reqs[0].rid)
        if rp is not None:
            seen.add(rp.fmt)
            if rp.fmt == "nvfp4":
                assert all(p >= eng.runner.kv.alloc.mix.P8 for p in rp.pages.values())
    assert eng.runner.promotions == 1 and seen == {"fp8", "nvfp4"}, (eng.runner.promotions, seen)
    assert len(reqs[0].output) == 6 and eng.runner.kv.alloc.used == 0
