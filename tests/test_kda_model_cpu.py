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


def _cached_engine(fmt: str, keep: int = 64) -> Engine:
    ecfg = EngineConfig(model="tiny_kda", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=64,
                        cuda_graphs=False, prefix_cache=bool(fmt), kda_state_cache=fmt, kda_state_cache_max=keep)
    return Engine(ecfg, model_config("tiny_kda"), max_seq=512)


def _two_turns(eng: Engine) -> tuple:
    """A 150-token first turn (prefill snapshots at 64 and 128), then a second turn whose prompt extends the first
    turn's prompt and output."""
    torch.manual_seed(11)
    p1 = torch.randint(1, 500, (150,)).tolist()
    o1 = eng.generate([p1], SamplingParams(max_new_tokens=6))[0]
    p2 = p1 + o1 + torch.randint(1, 500, (40,)).tolist()
    r2 = eng.add_request(p2, SamplingParams(max_new_tokens=6))
    while eng.has_work():
        eng.step()
    return o1, r2


def test_kda_state_cache_prefix_reuse_is_exact_in_fp32():
    """Hybrid-model prefix reuse: the second turn reuses the first turn's pages up to the deepest page boundary with
    a stored recurrent state (128 tokens here) and, with fp32 state rows, generates exactly what a cold engine does."""
    warm, cold = _cached_engine("fp32"), _cached_engine("")
    o1w, r2w = _two_turns(warm)
    o1c, r2c = _two_turns(cold)
    assert cold.runner.prefix_cache is None and r2c.cached_tokens == 0
    assert warm.runner.state_hits == 1 and r2w.cached_tokens == 128
    assert o1w == o1c and r2w.output == r2c.output


def test_kda_state_cache_quantized_rows_and_trim():
    """bf16 / fp8 state rows restore close to the fp32 state; the cache keeps at most kda_state_cache_max
    snapshots; an unknown state format is refused."""
    import pytest
    from inference_optimizations_b200.ops import kda as KD
    for fmt in ("bf16", "fp8"):
        eng = _cached_engine(fmt, keep=1)
        _, r2 = _two_turns(eng)
        assert eng.runner.state_hits == 1 and r2.cached_tokens == 128 and len(r2.output) == 6
        assert len(eng.runner.prefix_cache.states()) <= 1
        kv = eng.runner.kv
        row = 0
        kv.kda[0]["S"][row].normal_()
        ref = kv.kda[0]["S"][row].clone()
        snap = kv.snapshot_state(row, fmt)
        kv.reset_state(row)
        kv.restore_state(row, snap, fmt)
        err = ((kv.kda[0]["S"][row] - ref).norm() / ref.norm()).item()
        assert err < (0.01 if fmt == "bf16" else 0.05), (fmt, err)
        assert snap[0]["S"].shape[1] == KD.ROW_BYTES[fmt]
    with pytest.raises(ValueError):
        _cached_engine("nvfp4")


def test_kda_mtp_speculation_commit_fold_keeps_greedy_output():
    """MTP speculation on the hybrid model: a verify step runs each request's [pending, draft] through the KDA layers
    as two single-token updates and keeps the state after the first; a rejected draft sets the row back to it (the
    commit fold), so the emitted tokens are plain greedy decoding's.  Half of the drafts are scripted to the true
    next token so both the accepted and the rolled-back paths run."""
    torch.manual_seed(3)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (50, 13, 77)]

    def eng_(spec):
        ecfg = EngineConfig(model="tiny_kda", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=64,
                            cuda_graphs=False, prefix_cache=False, spec=spec, spec_policy="always")
        return Engine(ecfg, model_config("tiny_kda"), max_seq=256)
    plain = eng_(False).generate(prompts, SamplingParams(max_new_tokens=10))
    eng = eng_(True)
    run = eng.runner
    inner = run.spec_decode

    def scripted(reqs):
        for r in reqs:
            k = len(r.output)
            ref = plain[[p for p in prompts].index(r.prompt)]
            if k < len(ref) and k % 2 == 0:
                r.draft_state["d"] = ref[k]
        return inner(reqs)
    run.spec_decode = scripted
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=10))
    assert outs == plain
    acc = sum(r.accepted for r in eng.finished)
    steps = sum(r.spec_steps for r in eng.finished)
    assert 0 < acc < steps, (acc, steps)
