"""Data-parallel attention + expert-parallel MoE of the MLA family on 2 GPUs: every MoE layer goes through the
peer-memory exchange with grouped FP8 block-scaled GEMMs (`parallel/ep.py EPMoE`, one symmetric buffer shared by all
layers), rank 1 idles while rank 0 still prefills / decodes, and each rank's logits and greedy output equal a
one-GPU engine holding every expert.  Runs as two child processes (needs >= 2 GPUs)."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = textwrap.dedent("""
    import os, torch, torch.distributed as dist
    from inference_optimizations_b200.config import EngineConfig, model_config
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    spec = os.environ["DPEP_SPEC"] == "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    dev = f"cuda:{rank}"
    cfg = model_config("tiny_mla", expert_ffn=256, dense_ffn=512, weight_dtype="fp8", expert_dtype="fp8")
    prompts = [[(17 * i + 5 * j) % 500 + 1 for j in range(20 + 45 * i)] for i in range(4)]
    mine = [prompts[i] for i in ([0, 2, 3] if rank == 0 else [1])]
    def mk(ep):
        ecfg = EngineConfig(model="tiny_mla", device=dev, kv_dtype="nvfp4", max_running=4, chunked_prefill=32,
                            cuda_graphs=False, ep=ep, prefix_cache=False, spec=spec, spec_policy="always")
        return Engine(ecfg, cfg, max_seq=256, ep_rank=rank if ep > 1 else 0,
                      ep_group=dist.group.WORLD if ep > 1 else None)
    r1 = mk(1)
    eng = mk(world)
    # teacher-forced logits of one prompt per rank (both ranks score at once: the MoE exchanges are collective)
    p = mine[-1]
    la, lb = r1.runner.score(p), eng.runner.score(p)
    cos = torch.nn.functional.cosine_similarity(la, lb, dim=-1)
    top1 = (la.argmax(-1) == lb.argmax(-1)).float().mean().item()
    ref = r1.generate(mine, SamplingParams(max_new_tokens=6))
    got = eng.generate_dp(mine, SamplingParams(max_new_tokens=6))
    for ex in eng.runner.model.ep.values():
        ex.check()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    # the exchange moves bytes and the grouped GEMM + combine round at the same points as the one-GPU path, so the
    # logits and the greedy tokens match exactly (a random-init router has near-tie scores: any rounding difference
    # would flip experts)
    assert cos.min().item() > 0.9999 and top1 == 1.0, (rank, cos.min().item(), top1)
    assert got == ref, (rank, got, ref)
    print("rank", rank, "ok", cos.min().item(), top1, got, ref)
""")


@pytest.mark.parametrize("spec", [False, True])
def test_dp_ep_mla_two_gpus(cuda, tmp_path, spec):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "dpep_worker.py"
    script.write_text(WORKER)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT="29581" if not spec else "29582", DPEP_SPEC="1" if spec else "0",
                   NCCL_NVLS_ENABLE="0", PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
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
