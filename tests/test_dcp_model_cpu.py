"""Decode context parallelism inside the MLA model on CPU ranks (gloo): every rank runs the same tokens, writes only
the latent rows it owns, attends over them and merges the partial softmax states for its head group (collective
reference of the peer-memory merge); W_UV / W_o, the routed experts and the dense FFN columns are split over the
ranks and summed by an all-reduce.  The logits track a single-process model with the same weights, and both ranks
produce the same tokens."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_optimizations_b200.config import EngineConfig, model_config
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.scheduler import Request, SamplingParams, Segment

PROMPT = [(13 * j + 7) % 500 + 1 for j in range(150)]


def _engine(dcp: int, rank: int) -> Engine:
    ecfg = EngineConfig(model="tiny_mla", device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=64,
                        cuda_graphs=False, dcp=dcp, prefix_cache=False)
    return Engine(ecfg, model_config("tiny_mla"), max_seq=256, dcp_rank=rank,
                  dcp_group=dist.group.WORLD if dcp > 1 else None)


def _logits(eng: Engine) -> torch.Tensor:
    r = Request(rid=0, prompt=PROMPT, params=SamplingParams(max_new_tokens=1))
    r.slot = 0
    eng.runner.attach(r)
    st, _ = eng.runner._step([Segment(r, 0, PROMPT, True)])
    x = eng.runner.model.forward(st, eng.runner.kv)
    eng.runner.detach(r)
    return eng.runner.model.logits(x).float()


def _worker(rank: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        eng = _engine(2, rank)
        m = eng.runner.model
        assert m.layers[0].w_uv.shape[0] == model_config("tiny_mla").num_heads // 2
        # this rank's latent pool holds half the page space
        assert m.layers and eng.runner.kv.latent[0].shape[0] * 2 >= eng.runner.kv.index[0].shape[0] * 64
        logits = _logits(eng)
        outs = eng.generate([PROMPT[:70], PROMPT[:33]], SamplingParams(max_new_tokens=5))
        q.put((rank, logits, outs))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_dcp_model_matches_single_process():
    ref_logits = _logits(_engine(1, 0))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, logits, outs = q.get(timeout=600)
        got[rank] = (logits, outs)
    for p in procs:
        p.join(timeout=120)
    for rank in (0, 1):
        # split sums round differently from the single-process sums; a random-init router can flip a near-tie
        # expert on a rare token, so the bound is on the distribution, not the single worst token
        cos = torch.nn.functional.cosine_similarity(got[rank][0], ref_logits, dim=-1)
        assert cos.median().item() > 0.999 and (cos > 0.99).float().mean().item() > 0.95, (rank, cos)
    assert torch.equal(got[0][0], got[1][0])                 # the ranks hold identical activations
    assert got[0][1] == got[1][1]


def test_rank_index_ignored_without_context_parallelism():
    """A whole model built on a process whose rank is 1 (dcp_world 1) holds the shared expert and every head: the
    rank index only places work when context parallelism is on."""
    from inference_optimizations_b200.config import model_config
    from inference_optimizations_b200.models.mla import MLAModel
    cfg = model_config("tiny_mla")
    a = MLAModel(cfg, "cpu", 0, dcp_rank=1, dcp_world=1)
    b = MLAModel(cfg, "cpu", 0)
    i = cfg.first_dense
    assert a.layers[i].ffn["shared_gu"] is not None
    assert torch.equal(a.layers[i].ffn["shared_gu"], b.layers[i].ffn["shared_gu"])
