"""MLA + DSA + MoE model through the engine on CPU (every op's fp32 oracle path): chunked prefill + incremental
decode equals re-running the whole sequence, and the router oracle's rules."""
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams
from inference_optimizations_b200.ops import moe as MOE


def _engine(chunk=16, max_seq=256):
    ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=chunk,
                        cuda_graphs=False)
    return Engine(ecfg, model_config("tiny_mla"), max_seq=max_seq)


def test_mla_engine_incremental_matches_full_sequence():
    torch.manual_seed(0)
    cfg = model_config("tiny_mla")
    prompts = [torch.randint(0, cfg.vocab, (n,)).tolist() for n in (40, 70)]
    eng = _engine()
    out = eng.generate(prompts, SamplingParams(max_new_tokens=5))
    assert all(len(o) == 5 for o in out)
    # reference: each next token from a fresh engine prefilling the whole sequence in one chunk
    for p, o in zip(prompts, out):
        seq = list(p)
        for k in range(5):
            ref = _engine(chunk=512)
            nxt = ref.generate([seq], SamplingParams(max_new_tokens=1))[0][0]
            assert nxt == o[k], (k, nxt, o[k])
            seq.append(nxt)


def test_router_oracle_group_limits_and_weights():
    torch.manual_seed(1)
    t, e, k = 5, 16, 4
    logits = torch.randn(t, e)
    bias = torch.zeros(e)
    bias[3] = 5.0                                   # expert 3 always eligible for selection
    ids, w = MOE.route_ref(logits, bias, k, n_group=4, topk_group=2, routed_scale=2.5)
    assert (ids == 3).any(dim=1).all()
    groups = ids.long() // 4
    assert all(len(set(g.tolist())) <= 2 for g in groups)   # at most topk_group groups
    assert torch.allclose(w.sum(-1), torch.full((t,), 2.5))
    scores = torch.sigmoid(logits)
    assert torch.allclose(w / 2.5, scores.gather(1, ids.long()) / scores.gather(1, ids.long()).sum(-1, keepdim=True))


def test_radix_prefix_cache_reuse_is_exact():
    torch.manual_seed(5)
    cfg = model_config("tiny_mla")
    shared = torch.randint(0, cfg.vocab, (150,)).tolist()
    a = shared + torch.randint(0, cfg.vocab, (20,)).tolist()
    b = shared + torch.randint(0, cfg.vocab, (33,)).tolist()
    eng = _engine()
    out_a = eng.generate([a], SamplingParams(max_new_tokens=4))[0]
    held = eng.runner.prefix_cache.held
    assert held == (150 + 20 + 3) // 64                     # full pages of a's KV (prompt + 3 decoded tokens)
    r = eng.add_request(b, SamplingParams(max_new_tokens=4))
    while not r.finished:
        eng.step()
    assert eng.runner.prefix_cache.hits == 1
    # b reused 2 pages (128 tokens) of a's prefix; its tokens equal a cold engine's
    cold = _engine()
    cold.runner.prefix_cache = None
    assert r.output == cold.generate([b], SamplingParams(max_new_tokens=4))[0]
    # eviction frees unreferenced pages
    held, free0 = eng.runner.prefix_cache.held, eng.runner.kv.alloc.free
    assert eng.runner.prefix_cache.clear() == held and eng.runner.prefix_cache.held == 0
    assert eng.runner.kv.alloc.free == free0 + held


def test_mla_mtp_speculation_preserves_greedy_output():
    """Depth-1 MTP speculation (verify [pending, draft] in one target forward) emits exactly the plain greedy tokens;
    a draft that equals the target's next token is accepted (two tokens in one step)."""
    import torch
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    cfg = model_config("tiny_mla")
    torch.manual_seed(2)
    prompts = [torch.randint(1, cfg.vocab, (n,)).tolist() for n in (70, 21)]
    outs, engines = [], []
    for spec in (False, True):
        ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                            cuda_graphs=False, spec=spec, spec_policy="always", prefix_cache=False)
        eng = Engine(ecfg, cfg, max_seq=256)
        outs.append(eng.generate(prompts, SamplingParams(max_new_tokens=10)))
        engines.append(eng)
    assert outs[0] == outs[1], outs
    assert all(r.spec_steps > 0 for r in engines[1].finished)
    # forced acceptance: make the draft the target's own next token and check the step emits two tokens
    eng = engines[1]
    r = eng.add_request(prompts[1], SamplingParams(max_new_tokens=6))
    while r.prefilled < r.prompt_len:
        eng.step()
    plain = Engine(EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                                cuda_graphs=False, prefix_cache=False), cfg, max_seq=256)
    want = plain.generate([prompts[1]], SamplingParams(max_new_tokens=6))[0]
    r.draft_state["d"] = want[1]                    # the token greedy decoding produces after r.pending
    got = eng.runner.spec_decode([r])[r.rid]
    assert got == want[1:3], (got, want)


def test_synthetic_mla_sessions_decode():
    """Synthetic MLA sessions (pools filled through the writers) decode like any running request."""
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.synthetic import synth_mla_sessions
    ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=3, chunked_prefill=32,
                        cuda_graphs=False, prefix_cache=False)
    eng = Engine(ecfg, model_config("tiny_mla"), max_seq=256)
    reqs = synth_mla_sessions(eng, 3, 100, 4, seed=1)
    assert all(r.kv_len == 100 for r in reqs)
    out = eng.step()
    assert sorted(out) == sorted(r.rid for r in reqs) and all(len(v) == 1 for v in out.values())
