"""HTTP front end on CPU: /generate (single and batched), /health, /metrics, /flush_cache; the ranked front end over
data-parallel + expert-parallel ranks."""
import os
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


def _ranked_worker(rank: int, port: int, http_port: int, q):
    import torch.distributed as dist
    from inference_optimizations_b200.server.http import RankedEngineLoop, serve
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                            cuda_graphs=False, ep=2, prefix_cache=False)
        eng = Engine(ecfg, model_config("tiny_mla"), max_seq=256, ep_rank=rank, ep_group=dist.group.WORLD)
        loop = RankedEngineLoop(eng, rank, 2, dist.group.WORLD, "dp")
        if rank == 0:
            server, th, _ = serve(eng, port=http_port, block=False, loop=loop)
            q.put("up")
            loop.thread.join()
            server.should_exit = True
            th.join(timeout=5)
        else:
            loop.thread.join()
        q.put(("done", rank, loop.counters["steps"]))
    finally:
        dist.destroy_process_group()


def test_http_front_end_over_dp_ranks():
    """Rank 0's HTTP server feeds two data-parallel + expert-parallel ranks (gloo, CPU): the balancer spreads the
    prompts, the ranks step in lockstep, rank 0 answers with every output; the outputs equal one process's."""
    import torch.multiprocessing as mp
    prompts = [[(17 * i + 5 * j) % 500 + 1 for j in range(20 + 45 * i)] for i in range(4)]
    ref = Engine(EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                              cuda_graphs=False, prefix_cache=False), model_config("tiny_mla"),
                 max_seq=256).generate(prompts, SamplingParams(max_new_tokens=5))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, http_port = _free_port(), _free_port()
    procs = [ctx.Process(target=_ranked_worker, args=(r, port, http_port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        assert q.get(timeout=300) == "up"
        base = f"http://127.0.0.1:{http_port}"
        r = requests.post(base + "/generate", json={"prompts": prompts, "max_new_tokens": 5}, timeout=300)
        assert r.json()["outputs"] == ref
        m = requests.get(base + "/metrics", timeout=10).text
        assert "iob_requests_total 4" in m and 'iob_ttft_s{quantile="0.5"}' in m
        requests.post(base + "/shutdown", timeout=10)
        steps = dict((x[1], x[2]) for x in (q.get(timeout=120) for _ in range(2)))
        assert steps[0] == steps[1] > 0                       # lockstep
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
