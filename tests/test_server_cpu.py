"""HTTP front end on CPU: /generate (single and batched), /health, /metrics, /flush_cache."""
import socket

import requests

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import SamplingParams
from inference_optimizations_b200.server.http import serve


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_http_generate_matches_engine():
    mk = lambda: Engine(EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=4,  # noqa: E731
                                     chunked_prefill=32, cuda_graphs=False), model_config("tiny_gqa"), max_seq=128)
    prompts = [[1, 2, 3, 4, 5] * 4, [9, 8, 7] * 5]
    want = mk().generate(prompts, SamplingParams(max_new_tokens=4))
    port = _free_port()
    server, th, loop = serve(mk(), port=port, block=False)
    try:
        base = f"http://127.0.0.1:{port}"
        r = requests.post(base + "/generate", json={"input_ids": prompts[0], "max_new_tokens": 4}, timeout=60)
        assert r.json()["output_ids"] == want[0]
        r = requests.post(base + "/generate", json={"prompts": prompts, "max_new_tokens": 4}, timeout=60)
        assert r.json()["outputs"] == want
        assert requests.get(base + "/health", timeout=10).json()["ok"]
        m = requests.get(base + "/metrics", timeout=10).text
        assert "iob_requests_total 3" in m
        assert requests.post(base + "/flush_cache", timeout=10).json()["flushed"]
    finally:
        server.should_exit = True
        loop.shutdown()
        th.join(timeout=5)
