"""Process groups and the NCCL baseline collectives (one process per GPU, torch.distributed over NCCL).

`init()` reads RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR (torchrun) and creates the default NCCL group plus a gloo
group for host-side scheduler negotiation (the reference's CPU group for the prefill-delayer all-gather,
`scheduler/decode-burst/0004-*.patch`).  Every group gets a short timeout so ranks that wait on a dead peer end with an
error instead of hanging.  The collectives here are the measured baseline; the fused peer-memory kernels live in
`parallel/symm.py` and `csrc/comm.cu`.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    cpu_group: Optional[object] = None

    @property
    def enabled(self) -> bool:
        return self.world > 1


_INFO = DistInfo()


def init(backend: str = "nccl", timeout_s: float = 120.0) -> DistInfo:
    global _INFO
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        _INFO = DistInfo()
        return _INFO
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s)) if backend == "nccl" else None
    _INFO = DistInfo(rank, world, local, cpu)
    return _INFO


def info() -> DistInfo:
    return _INFO


def shutdown() -> None:
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def nccl_all_reduce(x: torch.Tensor) -> torch.Tensor:
    dist.all_reduce(x)
    return x


def host_all_reduce(x: torch.Tensor) -> torch.Tensor:
    """All-reduce for CPU tensors over gloo (fp32 accumulation, result cast back in place)."""
    xf = x.float()
    dist.all_reduce(xf)
    x.copy_(xf.to(x.dtype))
    return x


def argmax_merge(local_idx: torch.Tensor, local_val: torch.Tensor, vocab_local: int,
                 out: torch.Tensor) -> torch.Tensor:
    """Global greedy token from per-rank vocab-shard argmaxes: the max value, smallest global index on ties."""
    world = dist.get_world_size()
    if local_val.is_cuda:
        vals = torch.empty(world, local_val.numel(), dtype=local_val.dtype, device=local_val.device)
        idxs = torch.empty(world, local_idx.numel(), dtype=local_idx.dtype, device=local_idx.device)
        dist.all_gather_into_tensor(vals, local_val.contiguous())
        dist.all_gather_into_tensor(idxs, local_idx.contiguous())
    else:
        vl = [torch.empty_like(local_val) for _ in range(world)]
        il = [torch.empty_like(local_idx) for _ in range(world)]
        dist.all_gather(vl, local_val.contiguous())
        dist.all_gather(il, local_idx.contiguous())
        vals, idxs = torch.stack(vl), torch.stack(il)
    best = vals.argmax(dim=0)                       # first max = lowest rank = smallest global index
    g = torch.gather(idxs, 0, best[None]).squeeze(0) + best.to(idxs.dtype) * vocab_local
    out.copy_(g.to(out.dtype))
    return out


def max_over_ranks(x: float) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
