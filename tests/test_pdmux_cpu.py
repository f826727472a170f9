"""SM-partitioned prefill / decode lanes (engine/pdmux.py) on CPU: the pure rules, the split prefill reproducing the
plain engine's tokens, and the data-parallel lockstep (gloo ranks agree on every group and layer range)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_optimizations_b200.config import EngineConfig
from inference_optimizations_b200.engine.engine import Engine
from inference_optimizations_b200.engine.pdmux import PdmuxEngine, choose_group, divide_sms, split_layer_count
from inference_optimizations_b200.engine.scheduler import SamplingParams


def test_split_layer_count():
    assert split_layer_count([2048], 65536, 78, 0) == 32
    assert split_layer_count([2048, 0, 512], 65536, 78, 64) == 14     # the global max sets the range; clipped
    assert split_layer_count([0, 0], 65536, 78, 0) == 78               # every split idle: done at once
    assert split_layer_count([100000], 65536, 10, 3) == 1              # at least one layer
    assert split_layer_count([5], 1, 4, 4) == 0


def test_choose_group():
    assert choose_group(3, False, False, 0) == 0
    assert choose_group(3, False, True, 8) == 2
    assert choose_group(3, True, False, 0) == 0
    assert choose_group(3, True, True, 200) == 1
    assert choose_group(5, True, True, 0, decode_bs_divisor=36) == 1
    assert choose_group(5, True, True, 13, decode_bs_divisor=36) == 2
    assert choose_group(5, True, True, 500, decode_bs_divisor=36) == 3
    assert choose_group(5, True, True, 20, thresholds=(1, 16, 64)) == 2
    assert choose_group(5, True, True, 100, thresholds=(1, 16, 64)) == 3


def test_divide_sms():
    assert divide_sms(148, 3) == [(148, 0), (76, 72), (0, 148)]
    d = divide_sms(148, 5)
    assert [x[1] for x in d[1:-1]] == [40, 72, 112] and all(p + q == 148 for p, q in d[1:-1])


def _engine(max_running=4):
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=max_running, chunked_prefill=40,
                        cuda_graphs=False)
    return Engine(ecfg, max_seq=256)


PROMPTS = [list(range(3, 60)), list(range(7, 16)), list(range(100, 190)), list(range(1, 33))]


def test_pdmux_matches_plain_engine():
    params = SamplingParams(max_new_tokens=6)
    ref = _engine().generate(PROMPTS, params)
    pm = PdmuxEngine(_engine(), token_budget=40)          # 40-token chunks -> one layer per iteration
    outs = pm.generate(PROMPTS, params)
    assert outs == ref
    # the split spanned several iterations while decode steps ran beside it
    both = [e for e in pm.log if e[1] is not None and e[2] > 0]
    assert both and all(e[0] == 1 for e in both)
    assert any(e[1][1] - e[1][0] == 1 for e in pm.log if e[1] is not None)
    assert pm.engine.runner.kv.alloc["global"].used == 0


def _worker(rank: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        pm = PdmuxEngine(_engine(), token_budget=40, group=dist.group.WORLD)
        mine = PROMPTS if rank == 0 else PROMPTS[1:2]
        outs = pm.generate(mine, SamplingParams(max_new_tokens=6))
        q.put((rank, outs, pm.log))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_pdmux_dp_lockstep():
    params = SamplingParams(max_new_tokens=6)
    ref0 = _engine().generate(PROMPTS, params)
    ref1 = _engine().generate(PROMPTS[1:2], params)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (o, log)) for r, o, log in (q.get(timeout=600), q.get(timeout=600)))
    for p in procs:
        p.join(timeout=120)
    assert res[0][0] == ref0 and res[1][0] == ref1
    log0, log1 = res[0][1], res[1][1]
    assert len(log0) == len(log1)
    assert [(g, s) for g, s, _ in log0] == [(g, s) for g, s, _ in log1]   # same group and layer range every iteration


def test_engine_config_flag():
    """EngineConfig(pdmux=True): Engine.step / generate run through the lanes and give the plain tokens."""
    params = SamplingParams(max_new_tokens=5)
    ref = _engine().generate(PROMPTS, params)
    ecfg = EngineConfig(model="tiny_gqa", device="cpu", kv_dtype="bf16", max_running=4, chunked_prefill=40,
                        cuda_graphs=False, pdmux=True, pdmux_budget=40)
    eng = Engine(ecfg, max_seq=256)
    assert eng.generate(PROMPTS, params) == ref
    assert eng.pdmux.log and not eng.has_work()


@pytest.mark.parametrize("model", ["tiny_mla", "tiny_kda"])
def test_pdmux_mla_family_matches_plain_engine(model):
    """The MLA family (and the hybrid KDA + MLA model, whose recurrent states the split prefill carries) through the
    lanes: prefill split by layer ranges beside decode steps gives the plain engine's tokens, the split's last range
    ends with the LM head, pages are released."""
    from inference_optimizations_b200.config import model_config

    def mla_engine():
        ecfg = EngineConfig(model=model, device="cpu", kv_dtype="nvfp4", max_running=4, chunked_prefill=40,
                            cuda_graphs=False, prefix_cache=False)
        return Engine(ecfg, model_config(model), max_seq=256)
    params = SamplingParams(max_new_tokens=6)
    ref = mla_engine().generate(PROMPTS, params)
    pm = PdmuxEngine(mla_engine(), token_budget=40)          # 40-token chunks -> one layer per iteration
    outs = pm.generate(PROMPTS, params)
    assert outs == ref
    both = [e for e in pm.log if e[1] is not None and e[2] > 0]
    assert both
    assert any(e[1][1] - e[1][0] == 1 for e in pm.log if e[1] is not None)
    assert pm.engine.runner.kv.alloc.used == 0
