"""Expert-parallel MoE over peer memory (parallel/ep.py) on 2 GPUs: each rank's output equals the single-GPU
grouped-expert path on the same tokens with all experts local, for FP8 and NVFP4 weights, with an idle rank, and
across repeated layers (buffer reuse); the NCCL baseline exchange (`forward_nccl`) gives the same output bit for bit.  Runs as two child processes (needs >= 2 GPUs)."""
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
    from inference_optimizations_b200.parallel.ep import EPMoE
    from inference_optimizations_b200.ops import moe_gemm as MG
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    fmt = os.environ["EP_FMT"]
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    E, F, H, topk, T_max = 8, 256, 512, 3, 16
    g = torch.Generator().manual_seed(0)
    wg = torch.randn(E, F, H, generator=g) * 0.04
    wu = torch.randn(E, F, H, generator=g) * 0.04
    wd = torch.randn(E, H, F, generator=g) * 0.04
    sh = tuple(torch.randn(*s, generator=g) * 0.04 for s in ((F, H), (F, H), (H, F)))
    E_loc = E // world
    sl = slice(rank * E_loc, (rank + 1) * E_loc)
    ep = EPMoE(rank, world, E, T_max, topk, wg[sl].to(dev), wu[sl].to(dev), wd[sl].to(dev),
               shared=tuple(t.to(dev) for t in sh), fmt=fmt)
    full = MG.BlockScaledExperts(wg.to(dev), wu.to(dev), wd.to(dev), shared=tuple(t.to(dev) for t in sh), fmt=fmt)
    worst = 1.0
    for layer, T in enumerate([13, 16, 0 if rank == 1 else 7, 5]):
        gl = torch.Generator().manual_seed(100 + 10 * layer + rank)
        x = torch.randn(T, H, generator=gl).to(torch.bfloat16).to(dev)
        ids = torch.stack([torch.randperm(E, generator=gl)[:topk] for _ in range(T)]).int().to(dev) if T else \\
            torch.zeros(0, topk, dtype=torch.int32, device=dev)
        w = torch.softmax(torch.randn(T, topk, generator=gl), -1).to(dev)
        y = ep.forward(x, ids, w)
        torch.cuda.synchronize()
        ep.check()
        yn = ep.forward_nccl(x, ids, w)          # NCCL baseline exchange: the same values bit for bit
        torch.cuda.synchronize()
        if not torch.equal(y, yn):
            print(f"rank {rank} layer {layer}: NCCL path differs", flush=True)
            worst = -1.0
        if T:
            ref = full.forward(x, ids, w)
            cos = Fn.cosine_similarity(y.float().flatten(), ref.float().flatten(), dim=0).item()
            worst = min(worst, cos)
    print(f"rank {rank} worst_cos {worst:.6f}", flush=True)
    ok = worst > 0.999
    del ep
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)
""")


@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
def test_ep_moe_two_gpus(cuda, tmp_path, fmt):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "ep_worker.py"
    script.write_text(WORKER)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT="29571" if fmt == "fp8" else "29572", EP_FMT=fmt, NCCL_NVLS_ENABLE="0",
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
