"""Symmetric peer memory for the fused tensor-parallel collectives (csrc/comm.cu).

One buffer per TP group, allocated through torch's symmetric-memory rendezvous (CUDA virtual-memory allocations
exported to and mapped by every peer; no NVSHMEM): data halves [2][rows_cap][hidden] bf16 followed by [2][tp] int32
flags.  The row-parallel GEMMs write their partials straight into the current half (`out_buffer`), then one kernel
reduces over NVLink and applies the norm chain (`reduce_norm2`).  The reference moves the same kind of traffic with
its Triton push/pull kernels over torch symmetric memory (`moe-gemm/dp-moe-symmetric-memory/numinous_dp_moe.py:
89-141`); here the allocation is the only part taken from torch."""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .._ext import ext


class TPComm:
    def __init__(self, rank: int, world: int, rows_cap: int, hidden: int, device, group=None):
        import torch.distributed._symmetric_memory as symm
        self.rank, self.world, self.rows_cap, self.hidden = rank, world, rows_cap, hidden
        self.device = torch.device(device)
        data_bytes = 2 * rows_cap * hidden * 2
        self.flag_offset = data_bytes
        nbytes = data_bytes + ((2 * world * 4 + 255) // 256) * 256
        self.buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, grp)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.data = self.buf[:data_bytes].view(torch.bfloat16).view(2, rows_cap, hidden)
        self.epoch = torch.tensor([1, 0], dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.calls = 0
        torch.cuda.synchronize(self.device)
        dist.barrier(group=grp)          # every rank's flags are zero before anyone signals

    def out_buffer(self, rows: int) -> torch.Tensor:
        """[rows, hidden] view of the half the next reduce uses: the row-parallel GEMM writes its partial here."""
        if rows > self.rows_cap:
            raise ValueError(f"{rows} rows > capacity {self.rows_cap}")
        return self.data[self.calls % 2, :rows]

    def reduce_norm2(self, rows: int, resid: torch.Tensor, w1: Optional[torch.Tensor], w2: Optional[torch.Tensor],
                     eps: float, plus_one: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """o = rmsnorm(sum_r partial_r, w1); resid += o; return rmsnorm(resid, w2) (w1 / w2 None: skipped)."""
        if out is None:
            out = torch.empty_like(resid)
        ext().ar_norm2(self.peers, self.flag_offset, self.rows_cap, self.calls % 2, self.rank, self.epoch,
                       resid, out, w1, w2, eps, 1.0 if plus_one else 0.0, self.status)
        self.calls += 1
        return out

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError(f"peer-memory all-reduce: status {int(self.status.item())} (a peer did not arrive)")
