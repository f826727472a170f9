"""In-node prefill/decode disaggregation: KV pages move from the prefill engine's pool to the decode engine's pool over
NVLink (csrc/pd.cu), without a staging copy or a transfer library (the reference's one-launch CUDA-IPC copy,
`parallelism/in-node-pd-disaggregation/pd_nvlink_copy.py:1-30`, replacing Mooncake for same-node pairs).

Both engines of a pair map each other's pools through one symmetric allocation per side (torch symmetric-memory
rendezvous over the pair's group).  Protocol for one request:

  1. decode side reserves pages for the prompt in its allocator and sends their ids to the prefill side (host
     message: a store key or a gloo send; `PagePlan`);
  2. prefill side runs the prompt, then `push(src_pages, dst_pages, seq)` copies every layer's pages in one launch and
     publishes `seq` in the decode GPU's flag word (system-scope release after the copy);
  3. decode side enqueues `wait(seq)` on its forward stream (a bounded device wait, status on timeout) before the
     first decode step of the request, so no host round trip sits on the critical path.

Sequence numbers increase per transfer; the decode side's flag only grows, so one word serves every request.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .._ext import ext


@dataclass
class PagePlan:
    rid: int
    src_pages: list
    dst_pages: list
    seq: int


class PDPool:
    """One side's pool: [layers][pages * page_bytes] bytes + a flag word, in symmetric memory."""

    def __init__(self, layers: int, pages: int, page_bytes: int, device, group=None):
        import torch.distributed._symmetric_memory as symm
        self.layers, self.pages, self.page_bytes = layers, pages, page_bytes
        self.layer_stride = pages * page_bytes
        self.flag_off = layers * self.layer_stride
        self.buf = symm.empty(self.flag_off + 256, dtype=torch.uint8, device=device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, grp)
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.flag = self.buf[self.flag_off:self.flag_off + 4].view(torch.int32)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=grp)

    def layer(self, l: int) -> torch.Tensor:
        """[pages, page_bytes] view of layer l (what the attention kernels read as the pool)."""
        return self.buf[l * self.layer_stride:(l + 1) * self.layer_stride].view(self.pages, self.page_bytes)

    def push(self, peer: int, src_pages: list, dst_pages: list, seq: int) -> None:
        """Copy pages of every layer to the peer's pool and publish `seq` there (stream-ordered)."""
        dev = self.buf.device
        sp = torch.tensor(src_pages, dtype=torch.int32, device=dev)
        dp = torch.tensor(dst_pages, dtype=torch.int32, device=dev)
        ext().pd_copy(self.buf, self.ptrs[peer], sp, dp, self.page_bytes, self.layers, self.layer_stride,
                      self.layer_stride)
        ext().pd_signal(self.ptrs[peer] + self.flag_off, seq, self.buf)

    def wait(self, seq: int) -> None:
        """Device-side bounded wait until the peer published `seq` (enqueue before the step that reads the pages)."""
        ext().pd_wait(self.flag, seq, self.status)

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError("prefill->decode transfer: the prefill side did not publish in time")
