"""Fused GEMM -> all-reduce, push form (csrc/moe_gemm.cu broadcast epilogue + split-K reduction, csrc/comm.cu slot
sum): the GEMM's rows land in this rank's slot of every buffer of the peer table, bit-identical to the plain GEMM
output; the slot-sum reduce equals the pull-form reduce bit for bit; on 2 GPUs a tensor-parallel engine generates the
same tokens with the push form as with the pull form, and the NVLS form (switch-side reduction through the buffer's
multicast mapping) gives every rank the same rows, within bf16 rounding of the pull form.

One-GPU tests emulate the ranks with buffers on the same GPU (the peer table is just device pointers) and preset the
other rank's ready flag, so nothing waits on a rank that is not there."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

from inference_optimizations_b200.ops import linear as L

pytestmark = pytest.mark.gpu


class _LocalPush:
    """The `push_args` contract of a push-form TPComm over n local buffers, this rank = `rank`."""

    def __init__(self, n: int, rank: int, rows_cap: int, hidden: int, dev, half: int = 1):
        self.n, self.rank, self.rows_cap, self.hidden, self.half = n, rank, rows_cap, hidden, half
        self.bufs = [torch.full((2, n, rows_cap, hidden), -7.0, dtype=torch.bfloat16, device=dev) for _ in range(n)]
        self.peers = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device=dev)

    def push_args(self, rows: int):
        off = ((self.half * self.n + self.rank) * self.rows_cap) * self.hidden * 2
        return self.bufs[self.rank][self.half, self.rank, :rows], self.peers, off, self.n, self.rank


@pytest.mark.parametrize("kind", ["bf16", "fp8"])
@pytest.mark.parametrize("t", [1, 8, 37])
@pytest.mark.parametrize("ks", [1, 3])
def test_push_gemm_broadcasts_rows(cuda, kind, t, ks):
    torch.manual_seed(t + ks)
    N, K = 5376, 2688
    w = (torch.randn(N, K, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(t, K, device=cuda).to(torch.bfloat16)
    lin = L.Linear(w, kind)
    old = dict(L.FORCE)
    L.FORCE["ks"] = ks
    try:
        ref = lin(x).clone()
        p = _LocalPush(3, 1, 64, N, cuda)
        lin(x, push=p)
        torch.cuda.synchronize()
    finally:
        L.FORCE.update(old)
    for r, b in enumerate(p.bufs):
        assert torch.equal(b[1, 1, :t], ref), f"buffer {r}: pushed rows differ"
        assert bool((b[1, 1, t:] == -7.0).all()) and bool((b[0] == -7.0).all()) and bool((b[1, 0] == -7.0).all())
        assert bool((b[1, 2] == -7.0).all()), "only this rank's slot of the current half is written"


def test_slot_sum_reduce_equals_pull(cuda):
    """ar_norm2 in the push form (sum of the slots in this rank's buffer) == the pull form (each rank's own buffer,
    read through the peer table), bit for bit, for two emulated ranks on one GPU (rank 0 runs; rank 1's ready flag is
    preset)."""
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(0)
    T, H, cap, n = 19, 5376, 32, 2
    parts = [torch.randn(T, H, device=cuda).to(torch.bfloat16) for _ in range(n)]
    resid0 = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    w1 = (torch.randn(H, device=cuda) * 0.1).to(torch.bfloat16)
    w2 = (torch.randn(H, device=cuda) * 0.1).to(torch.bfloat16)
    outs = []
    for slots in (False, True):
        ns = n if slots else 1
        data = 2 * ns * cap * H * 2
        bufs = [torch.zeros(data + 256, dtype=torch.uint8, device=cuda) for _ in range(n)]
        for r in range(n):
            d = bufs[r][:data].view(torch.bfloat16).view(2, ns, cap, H)
            if slots:
                for q in range(n):
                    d[0, q, :T] = parts[q]           # every rank's push landed in every buffer
            else:
                d[0, 0, :T] = parts[r]               # each rank's own partial in its own buffer
        flags = bufs[0][data:data + 16].view(torch.int32)
        flags[1] = 1                                 # half 0, rank 1 arrived with value 1
        peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda)
        epoch = torch.tensor([1, 0], dtype=torch.int32, device=cuda)
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        resid = resid0.clone()
        out = torch.empty_like(resid)
        ext().ar_norm2(peers, data, cap, 0, 0, epoch, resid, out, w1, w2, 1e-6, 1.0, status, slots, 0, 0, 0)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        outs.append((resid, out))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


WORKER = textwrap.dedent("""
    import os, torch, torch.distributed as dist
    from inference_optimizations_b200.config import EngineConfig
    from inference_optimizations_b200.engine.engine import Engine
    from inference_optimizations_b200.engine.scheduler import SamplingParams
    from inference_optimizations_b200.parallel import dist as D
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    prompts = [[(13 * i + 7 * j) % 500 + 1 for j in range(30 + 25 * i)] for i in range(3)]
    res = {}
    for push in (False, True):
        ecfg = EngineConfig(model="tiny_gqa", device=f"cuda:{rank}", kv_dtype="bf16", max_running=4,
                            chunked_prefill=48, graph_batch_sizes="1,2,4", tp=world, tp_push=push)
        eng = Engine(ecfg, max_seq=256, tp_rank=rank, tp=world, all_reduce=D.nccl_all_reduce,
                     argmax_merge=D.argmax_merge)
        comm = eng.runner.tp_comm
        assert comm is not None and comm.push == push, (push, comm)
        res[push] = eng.generate(prompts, SamplingParams(max_new_tokens=6))
        torch.cuda.synchronize()
        comm.check()
        del eng
    assert res[True] == res[False], res
    if rank == 0:
        print("OK", res[True])
    dist.barrier()
    dist.destroy_process_group()
""")


def test_tp2_engine_push_equals_pull(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "w.py"
    script.write_text(WORKER)
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29531", WORLD_SIZE="2", NCCL_NVLS_ENABLE="0",
               PYTHONPATH=os.getcwd())
    procs = [subprocess.Popen([sys.executable, str(script)], env=dict(env, RANK=str(r)), stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = [p.communicate(timeout=600)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    assert "OK" in outs[0], outs


NVLS_WORKER = textwrap.dedent("""
    import os, torch, torch.distributed as dist
    from inference_optimizations_b200.parallel.symm import TPComm
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    H, cap = 5376, 64
    try:
        cn = TPComm(rank, world, cap, H, dev, nvls=True)
    except RuntimeError as e:
        ok = torch.zeros(1, device=dev)
    else:
        ok = torch.ones(1, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() == 0:
        if rank == 0:
            print("SKIP no multicast")
        dist.barrier(); dist.destroy_process_group(); raise SystemExit(0)
    cq = TPComm(rank, world, cap, H, dev)
    g = torch.Generator().manual_seed(0)
    w1 = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16).to(dev)
    w2 = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16).to(dev)
    worst = 0.0
    for T in (1, 7, 64):
        parts = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(world)]
        resid0 = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
        res = {}
        for name, c in (("pull", cq), ("nvls", cn)):
            resid = resid0.clone()
            for it in range(3):                                  # both halves, epochs advancing
                c.out_buffer(T).copy_(parts[rank].to(dev))
                x = c.reduce_norm2(T, resid, w1, w2, 1e-6)
            torch.cuda.synchronize()
            c.check()
            res[name] = (x.float(), resid.float())
        for a, b in zip(res["pull"], res["nvls"]):
            # the switch rounds the reduced bf16 pair sums its own way: within an ulp per call, relative to the rows
            worst = max(worst, (a - b).abs().max().item() / a.abs().max().item())
        allx = [torch.empty_like(res["nvls"][0]) for _ in range(world)]
        dist.all_gather(allx, res["nvls"][0])
        assert all(torch.equal(allx[0], a) for a in allx), "ranks differ"
    assert worst < 0.03, worst
    if rank == 0:
        print("OK", worst)
    dist.barrier()
    dist.destroy_process_group()
""")


def test_nvls_reduce_matches_pull_2gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "w.py"
    script.write_text(NVLS_WORKER)
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29533", WORLD_SIZE="2", PYTHONPATH=os.getcwd())
    procs = [subprocess.Popen([sys.executable, str(script)], env=dict(env, RANK=str(r)), stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    if "SKIP" in outs[0]:
        pytest.skip("no NVLink multicast mapping on this system")
    assert "OK" in outs[0], outs
