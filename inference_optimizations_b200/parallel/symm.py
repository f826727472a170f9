"""Symmetric peer memory for the fused tensor-parallel collectives (csrc/comm.cu).

One buffer per TP group, allocated through torch's symmetric-memory rendezvous (CUDA virtual-memory allocations
exported to and mapped by every peer; no NVSHMEM): data halves followed by [2][tp] int32 flags.

Pull form (`push=False`): data [2][rows_cap][hidden] bf16; the row-parallel GEMM writes its partial into the current
half of its own buffer (`out_buffer`), then one kernel reduces over NVLink (peer loads) and applies the norm chain
(`reduce_norm2`).

Push form (`push=True`, the fused GEMM -> all-reduce): data [2][tp][rows_cap][hidden]; the row-parallel GEMM on this
framework's kernel stores every finished output tile into slot `rank` of EVERY rank's buffer from its epilogue (the
split-K reduction does it when K is split), so the NVLink transfer runs under the remaining tiles' math; the reduce
kernel then sums the tp slots of its own buffer in rank order (local reads only) and applies the norm chain.  The
result is bit-identical to the pull form.  The reference's decode push path is the same idea over Triton kernels
(`moe-gemm/dp-moe-symmetric-memory/symm_collectives.py:330-363`).

NVLS form (`nvls=True`, NVSwitch systems whose symmetric allocation got an NVLink multicast mapping): partials as in
the pull form, then rank r reduces column shard r of every row inside the switch (`multimem.ld_reduce`) and
multicasts the reduced shard into every rank's reduced-rows area (`multimem.st`), so a rank moves one partial row out
and one reduced row in instead of (tp - 1) partial rows; layout: partials [2][rows_cap][hidden], reduced
[2][rows_cap][hidden], flags [2][tp], per-row flags [2][rows_cap][tp].  The reference moves the same kind of traffic with
its Triton push/pull kernels over torch symmetric memory (`moe-gemm/dp-moe-symmetric-memory/numinous_dp_moe.py:
89-141`); here the allocation is the only part taken from torch."""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .._ext import ext


class TPComm:
    def __init__(self, rank: int, world: int, rows_cap: int, hidden: int, device, group=None, push: bool = False,
                 nvls: bool = False):
        import torch.distributed._symmetric_memory as symm
        if push and nvls:
            raise ValueError("push and NVLS are two forms of the reduce; pick one")
        self.rank, self.world, self.rows_cap, self.hidden = rank, world, rows_cap, hidden
        self.push, self.nvls = push, nvls
        self.slots = world if push else 1
        self.device = torch.device(device)
        data_bytes = 2 * self.slots * rows_cap * hidden * 2
        self.res_offset = data_bytes                                  # NVLS: reduced rows after the partials
        if nvls:
            data_bytes *= 2
        self.flag_offset = data_bytes
        self.rowflag_offset = data_bytes + ((2 * world * 4 + 255) // 256) * 256
        nbytes = self.rowflag_offset + (((2 * rows_cap * world * 4 + 255) // 256) * 256 if nvls else 0)
        self.buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, grp)
        self.mc = int(self.handle.multicast_ptr) if nvls else 0
        if nvls and int(self.handle.buffer_ptrs[rank]) != self.buf.data_ptr():
            raise RuntimeError("NVLS reduce: the buffer does not start at its symmetric allocation's base")
        if nvls and not self.mc:
            raise RuntimeError("NVLS reduce: the symmetric buffer has no NVLink multicast mapping on this system")
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.data = self.buf[:2 * self.slots * rows_cap * hidden * 2].view(torch.bfloat16).view(
            2, self.slots, rows_cap, hidden)
        self.epoch = torch.tensor([1, 0], dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.calls = 0
        torch.cuda.synchronize(self.device)
        dist.barrier(group=grp)          # every rank's flags are zero before anyone signals

    def out_buffer(self, rows: int) -> torch.Tensor:
        """[rows, hidden] view of the half the next reduce uses: the row-parallel GEMM writes its partial here (pull
        form; in the push form this is only the local copy of this rank's slot)."""
        if rows > self.rows_cap:
            raise ValueError(f"{rows} rows > capacity {self.rows_cap}")
        return self.data[self.calls % 2, self.rank if self.push else 0, :rows]

    def push_args(self, rows: int) -> tuple:
        """Push form: (local view of this rank's slot [rows, hidden], peer table, byte offset of the slot inside
        every rank's buffer, ranks, rank) for the GEMM whose epilogue broadcasts its rows."""
        if not self.push:
            raise ValueError("push_args needs TPComm(push=True)")
        view = self.out_buffer(rows)
        off = (((self.calls % 2) * self.slots + self.rank) * self.rows_cap) * self.hidden * 2
        return view, self.peers, off, self.world, self.rank

    def reduce_norm2(self, rows: int, resid: torch.Tensor, w1: Optional[torch.Tensor], w2: Optional[torch.Tensor],
                     eps: float, plus_one: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """o = rmsnorm(sum_r partial_r, w1); resid += o; return rmsnorm(resid, w2) (w1 / w2 None: skipped)."""
        if out is None:
            out = torch.empty_like(resid)
        ext().ar_norm2(self.peers, self.flag_offset, self.rows_cap, self.calls % 2, self.rank, self.epoch,
                       resid, out, w1, w2, eps, 1.0 if plus_one else 0.0, self.status, self.push, self.mc,
                       self.res_offset, self.rowflag_offset)
        self.calls += 1
        return out

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError(f"peer-memory all-reduce: status {int(self.status.item())} (a peer did not arrive)")
