"""Engine end to end on CPU (torch oracle ops): paged prefill/decode must reproduce the cache-free reference."""
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams


def _engine(**kw):
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=4, chunked_prefill=40,
                        cuda_graphs=False, **kw)
    return Engine(ecfg, max_seq=256)


def test_prefill_decode_matches_reference():
    torch.manual_seed(0)
    eng = _engine()
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (57, 9, 100)]
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=6))
    for p, o in zip(prompts, outs):
        seq = list(p)
        for tok in o:
            ref = eng.runner.model.reference_logits(seq)[-1]
            top2 = torch.topk(ref, 2).values
            if (top2[0] - top2[1]).item() > 1e-2:      # skip numerically tied steps
                assert tok == int(ref.argmax()), (len(seq), tok, int(ref.argmax()))
            seq.append(tok)


def test_sliding_window_pages_released():
    eng = _engine()
    cfg = eng.cfg
    prompt = list(range(1, 200))
    eng.generate([prompt], SamplingParams(max_new_tokens=3))
    # after the request finished every page went back to the allocators
    assert eng.runner.kv.alloc["global"].used == 0
    assert eng.runner.kv.alloc["swa"].used == 0


def test_continuous_batching_many_requests():
    eng = _engine()
    prompts = [[5 + i] * (10 + 7 * i) for i in range(7)]       # more requests than max_running
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=4))
    assert all(len(o) == 4 for o in outs)


def test_speculative_decoding_preserves_greedy_output():
    torch.manual_seed(5)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (70, 33)]
    base = _engine().generate(prompts, SamplingParams(max_new_tokens=9))
    eng = _engine(spec=True, draft_tokens=3)
    spec = eng.generate(prompts, SamplingParams(max_new_tokens=9))
    ref_model = eng.runner.model
    for p, a, b in zip(prompts, base, spec):
        seq = list(p)
        for ta, tb in zip(a, b):
            ref = ref_model.reference_logits(seq)[-1]
            top2 = torch.topk(ref, 2).values
            if (top2[0] - top2[1]).item() <= 1e-2:
                break                      # numerically tied step: continuations may legitimately diverge
            assert ta == tb == int(ref.argmax())
            seq.append(ta)
    steps = [r for r in eng.finished]
    assert all(r.spec_steps > 0 for r in steps)


def test_spec_policy_math_and_switching():
    from inference_optimizations_b200.engine.spec_policy import SpecPolicy, expected_tokens, geometric_p
    assert geometric_p(0.0, 3) == 0.0 and geometric_p(3.0, 3) == 1.0
    p = geometric_p(1.5, 3)
    assert abs(p + p * p + p ** 3 - 1.5) < 1e-9
    assert expected_tokens(0.0, 4) == 1.0 and abs(expected_tokens(p, 4) - 2.5) < 1e-9
    # no acceptance: speculation (1.3x slower per step) loses -> plain decode until the running set changes
    pol = SpecPolicy(3, probe_steps=3)
    rids = [1, 2]
    modes = []
    for _ in range(8):
        spec = pol.use_spec(rids)
        modes.append(spec)
        if spec:
            pol.observe_spec(0.0, 1.3)
        else:
            pol.observe_plain(1.0)
    assert modes[:3] == [True] * 3 and not any(modes[3:])
    assert pol.history[-1]["spec"] is False
    assert pol.use_spec([1, 2, 3]) is True             # new running set: probe again
    # high acceptance: 2.5 tokens per 1.3x step beats plain
    pol = SpecPolicy(3, probe_steps=3)
    for _ in range(6):
        if pol.use_spec(rids):
            pol.observe_spec(1.5, 1.3)
        else:
            pol.observe_plain(1.0)
    assert pol.use_spec(rids) is True and pol.history[-1]["gain"] > 1.5
    assert SpecPolicy(3, "always").use_spec(rids) is True


def test_step_trace_records(tmp_path):
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    from inference_optimizations_b200.tooling.trace import read
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=2, chunked_prefill=16,
                        cuda_graphs=False, trace=str(tmp_path))
    eng = Engine(ecfg, model_config("tiny_gqa"), max_seq=128)
    eng.generate([[1, 2, 3] * 10, [4, 5] * 7], SamplingParams(max_new_tokens=3))
    eng.trace.flush()
    recs = read(str(tmp_path / "trace.rank0.jsonl"))
    assert len(recs) == len(eng.stats)
    assert {r["kind"] for r in recs} >= {"prefill", "decode"}
    assert all("schedule" in r["phases"] for r in recs) and recs[0]["step"] == 0


def test_scripted_drafts_control_acceptance():
    """Scripted drafts (the benchmark's controlled acceptance): when the script proposes the plain engine's own
    greedy continuation, every speculative step accepts all 3 drafts and the output is the plain output; when it
    proposes wrong tokens, none is accepted and the output is still the plain output."""
    torch.manual_seed(6)
    prompts = [torch.randint(1, 500, (n,)).tolist() for n in (40, 25)]
    params = SamplingParams(max_new_tokens=13)
    base = _engine().generate(prompts, params)
    for truth in (True, False):
        eng = _engine(spec=True, draft_tokens=3, spec_policy="always")
        reqs = [eng.add_request(p, params) for p in prompts]
        cont = {r.rid: list(p) + list(b) for r, p, b in zip(reqs, prompts, base)}

        def script(r, L, cont=cont, truth=truth):
            toks = [cont[r.rid][L + 1 + k] if L + 1 + k < len(cont[r.rid]) else 1 for k in range(3)]
            return [(t if truth else t % 499 + 1, True) for t in toks]
        eng.runner.draft_script = script
        while eng.has_work():
            eng.step()
        assert [r.output for r in reqs] == base
        acc = sum(r.accepted for r in reqs) / max(1, sum(r.spec_steps for r in reqs))
        assert (acc > 2.0) if truth else (acc == 0.0), acc
