"""FP8-quantized two-shot all-reduce over peer memory (csrc/qar.cu): about half the bytes of a bf16 all-reduce on
the wire, one quantization of each addend and one of the sum, results bitwise identical on every rank (the
reference's PCIe quantized all-reduce, `parallelism/fp8-pcie-allreduce/fp8_pcie_allreduce.py:1-30`).  For links
where bytes, not latency, bound the tensor-parallel all-reduce; on NVLink the fused bf16 all-reduce + norm
(`parallel/symm.py`) stays the default."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import ext


def _align(n: int) -> int:
    return (n + 255) // 256 * 256


class QuantAllReduce:
    def __init__(self, rank: int, world: int, T_max: int, H: int, device, group=None):
        import torch.distributed._symmetric_memory as symm
        assert H % 128 == 0
        self.rank, self.world, self.T_max, self.H = rank, world, T_max, H
        G = H // 128
        rq = world * T_max * G * 128
        rs = world * T_max * G * 4
        gq = T_max * G * 128
        gs = T_max * G * 4
        self.offs = [0, _align(rq), _align(rq) + _align(rs), _align(rq) + _align(rs) + _align(gq)]
        self.offs.append(self.offs[3] + _align(gs))
        nbytes = self.offs[4] + _align(2 * world * 4)
        self.buf = symm.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, grp)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=grp)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        ext().qar_allreduce(self.peers, self.offs, x.contiguous(), out, self.T_max, self.rank, self.world, self.epoch,
                            self.status)
        return out

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError("quantized all-reduce: a peer did not arrive")
