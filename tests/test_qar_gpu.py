"""FP8-quantized two-shot all-reduce (parallel/qar.py) on 2 GPUs: bitwise-identical results on both ranks, close to
the exact sum, repeated calls (epochs) and a smaller second shape.  Two child processes."""
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
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "qar_worker.py"
    script.write_text(WORKER)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT="29601", NCCL_NVLS_ENABLE="0",
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
