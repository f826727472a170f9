"""Session load generator + HTTP serving gate on CPU: the pure summary on hand-made turns, streamed multi-turn
sessions against a live tiny-model server (outputs equal the engine's own greedy generation of the same prompts),
and the A/B gate through HTTP with in-process servers."""
import socket

import pytest
import torch

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams
from inference_optimizations_b200.tooling import session_bench as SB


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_summary_math():
    spec = SB.SessionSpec(sessions=2, turns=2, prefix=10, question=2, output=5)
    rs = [SB.TurnResult(0, 1, 10, 0, 5, 0.5, 1.0, 0.0), SB.TurnResult(1, 1, 10, 0, 5, 0.4, 1.0, 0.0),
          SB.TurnResult(0, 2, 17, 10, 5, 0.1, 0.5, 1.0), SB.TurnResult(1, 2, 17, 0, 5, 0.3, 1.3, 1.0)]
    s = SB.summarize(rs, spec)
    assert s["sessions_completed"] == 2 and s["requests_ok"] == 4
    assert s["warm"]["agg_out_tok_s"] == pytest.approx(10 / 1.3, abs=1e-3)         # 10 tokens over [1.0, 2.3]
    assert s["warm"]["hit_rate"] == pytest.approx(10 / 34, abs=1e-4)
    assert s["warm"]["per_user_tok_s"]["p50"] == pytest.approx(4 / 1.0, abs=1e-3)  # rates 10.0 and 4.0
    assert s["warm"]["per_user_tok_s"]["p99"] == pytest.approx(4 / 1.0, abs=1e-3)
    assert s["cold"]["prefill_tok_s"] == pytest.approx(20 / 0.5, abs=1e-3)
    assert s["warm"]["ttft_s"]["max"] == pytest.approx(0.3)


def _engine():
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=4, chunked_prefill=64,
                        cuda_graphs=False)
    return Engine(ecfg, model_config("tiny_gqa"), max_seq=512)


def test_streamed_sessions_against_live_server():
    from inference_optimizations_b200.server.http import serve
    torch.manual_seed(0)
    port = _port()
    server, th, loop = serve(_engine(), port=port, block=False)
    try:
        spec = SB.SessionSpec(sessions=3, turns=3, prefix=40, question=6, output=4, vocab=500, seed=1)
        import asyncio
        res = asyncio.run(SB.run(f"http://127.0.0.1:{port}", spec))
        s = SB.summarize(res, spec)
    finally:
        loop.shutdown()
        server.should_exit = True
        th.join(timeout=10)
    assert s["requests_failed"] == 0 and s["requests_ok"] == 9 and s["sessions_completed"] == 3
    assert all(r.completion_tokens == 4 and 0 < r.ttft_s <= r.wall_s for r in res)
    assert s["warm"]["prompt_tokens_mean"] == pytest.approx((50 + 60) / 2)
    # the server's greedy outputs are the engine's: replay session 0's turns directly
    ref = _engine()
    import random
    rng = random.Random(spec.seed * 1_000_003 + 0)
    prompt = [rng.randrange(1, spec.vocab) for _ in range(spec.prefix)]
    turns = sorted([r for r in res if r.session == 0], key=lambda r: r.turn)
    for r in turns:
        out = ref.generate([prompt], SamplingParams(max_new_tokens=spec.output))[0]
        assert r.prompt_tokens == len(prompt) and r.tokens == out
        prompt = prompt + out + [rng.randrange(1, spec.vocab) for _ in range(spec.question)]


def test_http_gate_in_process():
    from inference_optimizations_b200.server.http import serve
    from inference_optimizations_b200.tooling.serving_gate import gate_http

    def launcher():
        port = _port()
        server, th, loop = serve(_engine(), port=port, block=False)

        def stop():
            loop.shutdown()
            server.should_exit = True
            th.join(timeout=10)
        return f"http://127.0.0.1:{port}", stop

    spec = SB.SessionSpec(sessions=2, turns=2, prefix=24, question=4, output=3, vocab=500)
    res = gate_http({"control": launcher, "delta": launcher}, spec, repeats=2, delta={"note": "same engine"})
    assert res["verdict"] in ("neutral", "better", "worse")
    for arm in ("control", "delta"):
        runs = res["arms"][arm]["runs"]
        assert len(runs) == 2 and all(r["requests_failed"] == 0 and r["sessions_completed"] == 2 for r in runs)
