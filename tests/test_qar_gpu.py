"""FP8-quantized two-shot all-reduce (parallel/qar.py) on 2 GPUs: bitwise-identical results on both ranks, close to
the exact sum, repeated calls (epochs) and a smaller second shape; and as the tensor-parallel engine's all-reduce
(`EngineConfig.tp_qar`): every step's reduce through it, status clean, greedy tokens close to the exact reduce's.  Two
child processes per test."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = textwrap.dedent("""
    import os, sys, torch, torch.distributed as dist
    import torch.nn.functional as Fn
    from inference_optimizations_b200.parallel.qar import QuantAllReduce
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    qar = QuantAllReduce(rank, world, 64, 5376, dev)
    ok = True
    for it, T in enumerate([37, 64, 5, 37]):
        g = torch.Generator().manual_seed(10 * it)
        xs = [torch.randn(T, 5376, generator=g).to(torch.bfloat16) for _ in range(world)]
        y = qar(xs[rank].to(dev))
        torch.cuda.synchronize()
        qar.check()
        exact = sum(x.float() for x in xs)
        cos = Fn.cosine_similarity(y.float().cpu().flatten(), exact.flatten(), dim=0).item()
        allv = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(allv, y)
        same = all(torch.equal(allv[0], v) for v in allv)
        ok = ok and same and cos > 0.998
        print(f"rank {rank} it {it} cos {cos:.5f} identical {same}", flush=True)
    del qar
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)
""")


def test_quantized_allreduce_two_gpus(cuda, tmp_path):
    _run_pair(tmp_path, WORKER, "29601")


ENGINE_WORKER = textwrap.dedent("""
    import os, sys, torch, torch.distributed as dist
    from inference_optimizations_b200.config import EngineConfig
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    from inference_optimizations_b200.parallel import dist as D
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    prompts = [[(13 * i + 7 * j) % 500 + 1 for j in range(30 + 25 * i)] for i in range(3)]
    res = {}
    for qar in (False, True):
        ecfg = EngineConfig(model="tiny_gqa", device=f"cuda:{rank}", kv_dtype="bf16", max_running=4,
                            chunked_prefill=48, graph_batch_sizes="1,2,4", tp=world, tp_qar=qar, fused_comm=not qar)
        eng = Engine(ecfg, max_seq=256, tp_rank=rank, tp=world, all_reduce=D.nccl_all_reduce,
                     argmax_merge=D.argmax_merge)
        assert (eng.runner.qar is not None) == qar and (eng.runner.tp_comm is None) == qar
        res[qar] = eng.generate(prompts, SamplingParams(max_new_tokens=6))
        torch.cuda.synchronize()
        if qar:
            eng.runner.qar.check()
        del eng
    agree = sum(a == b for x, y in zip(res[True], res[False]) for a, b in zip(x, y)) / 18
    first = all(x[0] == y[0] for x, y in zip(res[True], res[False]))
    print(f"rank {rank} qar vs exact reduce: token agreement {agree:.3f} first {first}", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    # lossy reduce (E4M3 addends and sum): the first tokens, and most later ones, match the exact reduce's
    sys.exit(0 if first and agree >= 0.6 else 1)
""")


def test_tp2_engine_quantized_allreduce(cuda, tmp_path):
    _run_pair(tmp_path, ENGINE_WORKER, "29602")


def _run_pair(tmp_path, worker: str, port: str):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "qar_worker.py"
    script.write_text(worker)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=port, NCCL_NVLS_ENABLE="0",
                   PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for p, out in zip(procs, outs):
        assert p.returncode == 0, out[-3000:]
