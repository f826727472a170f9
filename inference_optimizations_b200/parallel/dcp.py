"""Decode context parallelism (DCP) for sparse-MLA (DSA) decode: the latent KV of a sequence is sharded over S GPUs by
the owner rule, every rank attends over the selected rows it owns, and the partial softmax states are merged over
NVLink peer memory (csrc/dcp.cu).

Owner rule (`parallelism/dsa-decode-context-parallel/dcp_topk.py:3-9`): virtual pool row v lives on rank v % S at local
row v // S, so a sequence's pages interleave over the group and each rank holds 1/S of every context.  The indexer
key cache stays replicated over the virtual rows (`parallelism/README.md:7`), so every rank computes the same full
top-k; `owned_local_rows` turns it into local rows (-1 where another rank owns the row, no compaction, as the
reference's `_dcp_owned_in_place`).  `select_dcp` is the sharded-key alternative: local top-k, all-gather of S x k
candidates, global top-k of the union (`dcp_topk.py:30-80`).

Merge: rank r keeps head group r (heads [r H / S, (r + 1) H / S)), the input of a row-parallel o_proj whose partial
sums then go through the fused all-reduce; it pulls only its heads of every peer's (o, lse) -- 1/S of each partial
crosses NVLink instead of an all-gather of whole partials.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .._ext import ext


def owner(v: torch.Tensor, S: int) -> torch.Tensor:
    return v % S


def local_row(v: torch.Tensor, S: int) -> torch.Tensor:
    return v // S


def owned_local_rows(sel: torch.Tensor, rank: int, S: int) -> torch.Tensor:
    """Virtual rows [T, K] (-1 = masked) -> this rank's local rows where it owns them, -1 elsewhere."""
    own = (sel >= 0) & (sel % S == rank)
    return torch.where(own, sel // S, torch.full_like(sel, -1))


def merge_topk(scores: torch.Tensor, rows: torch.Tensor, k: int) -> torch.Tensor:
    """Union of candidates [B, C] (score, virtual row; row -1 = no candidate) -> the k best rows per query (ties: lower
    row first), -1 padded."""
    s = torch.where(rows >= 0, scores, torch.full_like(scores, float("-inf")))
    big = rows.max().clamp(min=0) + 1
    key_rows = torch.where(rows >= 0, rows, big)
    order = torch.sort(key_rows, dim=-1, stable=True).indices           # lower row first, then stable by score
    s_sorted, r_sorted = s.gather(1, order), rows.gather(1, order)
    top = torch.sort(s_sorted, dim=-1, descending=True, stable=True).indices[:, :k]
    out = r_sorted.gather(1, top)
    return torch.where(s_sorted.gather(1, top) == float("-inf"), torch.full_like(out, -1), out)


def select_dcp(local_scores: torch.Tensor, local_rows: torch.Tensor, k: int,
               all_gather: Optional[Callable] = None) -> torch.Tensor:
    """Sharded-key selection: local top-k over this rank's candidates -> gather of every rank's k candidates -> global
    top-k.  local_scores / local_rows [B, N_local] (rows are virtual rows, -1 = none).  `all_gather(t) -> list` of
    every rank's tensor (default: torch.distributed)."""
    kk = min(k, local_scores.shape[1])
    s = torch.where(local_rows >= 0, local_scores, torch.full_like(local_scores, float("-inf")))
    top = torch.sort(s, dim=-1, descending=True, stable=True).indices[:, :kk]
    cand_s, cand_r = s.gather(1, top), local_rows.gather(1, top)
    if all_gather is None:
        def all_gather(t):
            out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
            dist.all_gather(out, t)
            return out
    ss, rr = torch.cat(all_gather(cand_s), dim=1), torch.cat(all_gather(cand_r), dim=1)
    return merge_topk(ss, rr, k)


def merge_partials_ref(os: list, lses: list) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 oracle of the merge: partials o_s [T, H, D] with natural-log lse_s [T, H] (-inf: empty)."""
    lse = torch.stack([l.float() for l in lses])                        # [S, T, H]
    m = lse.max(0).values
    safe_m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(lse - safe_m)
    w = torch.where(torch.isfinite(lse), w, torch.zeros_like(w))
    den = w.sum(0)
    o = sum(w[i][..., None] * os[i].float() for i in range(len(os)))
    o = torch.where(den[..., None] > 0, o / den.clamp(min=1e-30)[..., None], torch.zeros_like(o))
    return o, torch.where(den > 0, safe_m + torch.log(den.clamp(min=1e-30)), torch.full_like(den, float("-inf")))


class DCPAttention:
    """Symmetric buffer: two halves of (o bf16 [T_max, H, 512], lse fp32 [T_max, H]) followed by flags [2][S]."""

    def __init__(self, rank: int, S: int, T_max: int, H: int, device, group=None):
        import torch.distributed._symmetric_memory as symm
        self.rank, self.S, self.T_max, self.H = rank, S, T_max, H
        self.Hg = H // S
        self.device = torch.device(device)
        self.half_bytes = T_max * H * (512 * 2 + 4)
        self.off_flags = 2 * self.half_bytes
        nbytes = self.off_flags + ((2 * S * 4 + 255) // 256) * 256
        self.buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, grp)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.epoch = torch.tensor([1, 0], dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.calls = 0
        torch.cuda.synchronize(self.device)
        dist.barrier(group=grp)

    def partial_views(self, T: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(o [T, H, 512] bf16, lse [T, H] fp32) of the half the next merge reads: the decode kernel writes here."""
        base = (self.calls % 2) * self.half_bytes
        o = self.buf[base:base + self.T_max * self.H * 1024].view(torch.bfloat16).view(self.T_max, self.H, 512)
        lb = base + self.T_max * self.H * 1024
        lse = self.buf[lb:lb + self.T_max * self.H * 4].view(torch.float32).view(self.T_max, self.H)
        return o[:T], lse[:T]

    def merge(self, T: int, out: Optional[torch.Tensor] = None, lse_out: Optional[torch.Tensor] = None):
        """Merge the S partials of the current half for this rank's head group -> bf16 [T, Hg, 512]."""
        if out is None:
            out = torch.empty(T, self.Hg, 512, dtype=torch.bfloat16, device=self.device)
        if T == 0:
            return out
        ext().dcp_merge(self.peers, 0, self.off_flags, T, self.T_max, self.H, self.rank, self.S, self.calls % 2,
                        self.epoch, out, lse_out, self.status)
        self.calls += 1
        return out

    def decode(self, q: torch.Tensor, local_pool: torch.Tensor, sel: torch.Tensor, sm_scale: float, fmt: int,
               lse_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """q bf16 [T, H, 576]; sel int32 [T, K] virtual rows (the replicated indexer's top-k) -> merged o of this
        rank's head group [T, Hg, 512]."""
        from ..ops import mla as M
        T = q.shape[0]
        o, lse = self.partial_views(T)
        local = owned_local_rows(sel, self.rank, self.S).int()
        if T:
            M.mla_decode(q, local_pool, local, sm_scale, fmt, out=o, lse=lse, return_lse=True)
        return self.merge(T, lse_out=lse_out)

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError(f"DCP merge: status {int(self.status.item())} (a peer did not arrive)")


class DCPAttentionRef:
    """Collective reference of `DCPAttention` for any backend (gloo on CPU): each rank decodes over the rows it owns,
    the (o, lse) partials of every rank are all-gathered and merged in fp32 (`merge_partials_ref`), and the rank keeps
    its head group -- the same inputs and outputs as the peer-memory path."""

    def __init__(self, rank: int, S: int, H: int, group=None):
        self.rank, self.S, self.H, self.Hg, self.group = rank, S, H, H // S, group

    def decode(self, q: torch.Tensor, local_pool: torch.Tensor, sel: torch.Tensor, sm_scale: float, fmt: int,
               lse_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        from ..ops import mla as M
        local = owned_local_rows(sel, self.rank, self.S).int()
        o, lse = M.mla_decode(q, local_pool, local, sm_scale, fmt, return_lse=True)
        os_ = [torch.empty_like(o, dtype=torch.float32) for _ in range(self.S)]
        ls = [torch.empty_like(lse) for _ in range(self.S)]
        dist.all_gather(os_, o.float().contiguous(), group=self.group)
        dist.all_gather(ls, lse.contiguous(), group=self.group)
        om, lm = merge_partials_ref(os_, ls)
        g0 = self.rank * self.Hg
        if lse_out is not None:
            lse_out.copy_(lm[:, g0:g0 + self.Hg])
        return om[:, g0:g0 + self.Hg].to(torch.bfloat16)

    def check(self) -> None:
        pass
