"""Context-parallel sparse-MLA decode on 2 GPUs (parallel/dcp.py + csrc/dcp.cu): each rank decodes over the rows
it owns and merges the partial softmax states of its head group over peer memory; the result matches the
single-GPU decode over the whole pool (same E4M3 kernel), over repeated calls (both buffer halves) and with tokens
whose selection a rank does not own at all.  Two child processes (needs >= 2 GPUs)."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = textwrap.dedent("""
    import math, os, sys, torch, torch.distributed as dist
    import torch.nn.functional as Fn
    from inference_optimizations_b200.parallel.dcp import DCPAttention
    from inference_optimizations_b200.ops import mla as M
    from inference_optimizations_b200.utils.microbench import mla_pool_random
    rank, S = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    T_max, H, N, K = 8, 128, 8192, 640
    fmt = M.FMT_NVFP4
    pool = mla_pool_random(N, fmt, dev, seed=7)                 # identical on both ranks (seeded)
    local = pool[rank::S].contiguous()
    dc = DCPAttention(rank, S, T_max, H, dev)
    sm = 1.0 / math.sqrt(576)
    worst = 1.0
    for it, T in enumerate([5, 8, 3]):
        g = torch.Generator().manual_seed(10 + it)
        q = (torch.randn(T, H, 576, generator=g) * 0.5).to(torch.bfloat16).to(dev)
        sel = torch.stack([torch.randperm(N, generator=g)[:K] for _ in range(T)]).int()
        sel[0, K // 2:] = -1
        if T > 2:
            sel[2] = torch.arange(K, dtype=torch.int32) * S            # token 2: rank 0 owns every row
        sel = sel.to(dev)
        o = dc.decode(q, local, sel, sm, fmt)
        ref = M.mla_decode(q, pool, sel, sm, fmt)[:, rank * (H // S):(rank + 1) * (H // S)]
        torch.cuda.synchronize()
        dc.check()
        cos = Fn.cosine_similarity(o.float().flatten(), ref.float().flatten(), dim=0).item()
        err = ((o.float() - ref.float()).norm() / ref.float().norm()).item()
        worst = min(worst, cos)
        print(f"rank {rank} it {it} cos {cos:.6f} rel {err:.4f}", flush=True)
    ok = worst > 0.999
    del dc
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)
""")


def test_dcp_decode_two_gpus(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "dcp_worker.py"
    script.write_text(WORKER)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT="29581", NCCL_NVLS_ENABLE="0",
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


MODEL_WORKER = textwrap.dedent("""
    import os, sys, torch, torch.distributed as dist
    import torch.nn.functional as Fn
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import Request, SamplingParams, Segment
    rank, S = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    wdt = os.environ["DCP_WDT"]
    over = dict(expert_ffn=256, dense_ffn=512, weight_dtype=wdt, expert_dtype=wdt, hidden=512, q_lora=256,
                qk_nope=128, v_head=128, index_heads=8, num_heads=8)
    cfg = model_config("tiny_mla", **over)
    prompt = [(13 * j + 7) % 500 + 1 for j in range(150)]

    def logits(eng):
        r = Request(rid=0, prompt=prompt, params=SamplingParams(max_new_tokens=1))
        r.slot = 0
        eng.runner.attach(r)
        st, _ = eng.runner._step([Segment(r, 0, prompt, True)])
        x = eng.runner.model.forward(st, eng.runner.kv)
        eng.runner.detach(r)
        return eng.runner.model.logits(x).float()

    def engine(dcp):
        ecfg = EngineConfig(model="tiny_mla", device=str(dev), kv_dtype="nvfp4", max_running=4, chunked_prefill=256,
                            cuda_graphs=False, dcp=dcp, prefix_cache=False)
        return Engine(ecfg, cfg, max_seq=256, dcp_rank=rank, dcp_group=dist.group.WORLD if dcp > 1 else None)
    ref = logits(engine(1))                      # the whole model on this GPU (same seeded weights)
    eng = engine(S)
    got = logits(eng)
    outs = eng.generate([prompt[:70], prompt[:33]], SamplingParams(max_new_tokens=5))
    torch.cuda.synchronize()
    eng.runner.model.dcp.check()
    eng.runner.model.dcp_comm.check()
    cos = Fn.cosine_similarity(got, ref, dim=-1)
    # identical activations on both ranks, greedy tokens included
    both = [torch.empty_like(got) for _ in range(S)]
    dist.all_gather(both, got.contiguous())
    same = torch.equal(both[0], both[1])
    print(f"rank {rank} cos median {cos.median().item():.5f} min {cos.min().item():.5f} same {same} {outs}",
          flush=True)
    # The context-parallel model sums bf16 partials (row-parallel W_UV / W_o, split FFN) where the one-GPU model
    # accumulates once, and each rank's sparse attention rounds P to E4M3 against its own running max; a random-init
    # router can flip a near-tie expert on a rare token (measured with bf16 weights: median 0.9995, minimum 0.943).
    med, lo = 0.99, 0.9
    ok = cos.median().item() > med and cos.min().item() > lo and same
    dist.barrier()
    del eng
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)
""")


@pytest.mark.parametrize("wdt", ["bf16", "fp8"])
def test_dcp_model_two_gpus(cuda, tmp_path, wdt):
    """The MLA model with decode context parallelism on 2 GPUs (owned latent rows, peer-memory merge, fused
    all-reduce + norm of the row-parallel products) tracks the whole model on one GPU; both ranks agree exactly."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "dcp_model_worker.py"
    script.write_text(MODEL_WORKER)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT="29583" if wdt == "bf16" else "29584", NCCL_NVLS_ENABLE="0", DCP_WDT=wdt,
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
