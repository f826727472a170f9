"""Sparse MLA (DSA) decode over the compressed latent pool: csrc/attn_mla_decode.cu and its fp32 oracle.

Semantics of the reference's sparse FP4 decode (`kv-cache-4bit/glm-kv4/glm_kv4.py:575-622` `sparse_mla`, the native
`kv-cache-4bit/kv4mla/csrc/api.cpp:73` `sparse_decode`): query token t (H heads x 576 = 512 latent + 64 rope) attends to
the pool rows idx[t, :] (-1 = masked); K = the full row, V = its 512 latent values; returns out [T, H, 512] and the
natural-log LSE [T, H].  Rows are NVFP4 352-B rows (FMT_NVFP4) or E4M3 576-B rows (FMT_FP8)."""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from .._ext import ext
from . import formats as F
from .kvcache import FMT_FP8, FMT_NVFP4

NUM_SMS = 148
TILE = 128
ROW_BYTES = {FMT_NVFP4: F.MLA_ROW_BYTES, FMT_FP8: F.MLA_FP8_ROW_BYTES}


def mla_split_policy(tokens: int, topk: int, overhead_tiles: float = 2.0) -> tuple[int, int]:
    """(num_splits, tiles_per_split) for `tokens` query tokens over a top-k list of `topk` rows.  Each token runs
    two CTAs (one per V half); one CTA per SM at a time.  Minimises waves x (tiles per split + fixed overhead) plus
    the combine pass.  Depends only on (tokens, topk), so a captured graph keeps a valid schedule."""
    tiles = max(1, -(-topk // TILE))
    best, best_cost = 1, None
    for s in range(1, min(tiles, 64) + 1):
        ctas = 2 * tokens * s
        waves = -(-ctas // NUM_SMS)
        tps = -(-tiles // s)
        cost = waves * (tps + overhead_tiles) + (0.75 if s > 1 else 0.0)
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    tps = -(-tiles // best)
    return -(-tiles // tps), tps


@dataclass
class MlaWorkspace:
    o_part: torch.Tensor
    lse_part: torch.Tensor
    status: torch.Tensor

    @staticmethod
    def allocate(tokens: int, heads: int, max_splits: int, device="cuda") -> "MlaWorkspace":
        n = max(1, tokens * heads * max_splits)
        return MlaWorkspace(torch.empty(n * 512, dtype=torch.float32, device=device),
                            torch.empty(n, dtype=torch.float32, device=device),
                            torch.zeros(1, dtype=torch.int32, device=device))


def mla_decode(q: torch.Tensor, pool: torch.Tensor, idx: torch.Tensor, sm_scale: float, fmt: int = FMT_NVFP4,
               splits: Optional[tuple[int, int]] = None, ws: Optional[MlaWorkspace] = None,
               out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
               return_lse: bool = False):
    """q bf16 [T, H, 576], pool uint8 [rows, 352 | 576], idx int32 [T, topk] -> out bf16 [T, H, 512]
    (and lse fp32 [T, H], natural log, with return_lse)."""
    t, h, _ = q.shape
    if out is None:
        out = torch.empty(t, h, F.MLA_NOPE, dtype=torch.bfloat16, device=q.device)
    if return_lse and lse is None:
        lse = torch.empty(t, h, dtype=torch.float32, device=q.device)
    if not q.is_cuda:
        o, l = mla_decode_ref(q, pool, idx, sm_scale, fmt)
        out.copy_(o.to(out.dtype))
        if lse is not None:
            lse.copy_(l)
        return (out, lse) if return_lse else out
    if splits is None:
        splits = mla_split_policy(t, idx.shape[1])
    ns, tps = splits
    if ws is None:
        ws = MlaWorkspace.allocate(t, h, ns, device=q.device)
    ext().mla_decode(q, pool, idx, out, lse, ws.o_part, ws.lse_part, ws.status, fmt, tps, ns, sm_scale)
    return (out, lse) if return_lse else out


def dequant_rows(pool: torch.Tensor, fmt: int) -> torch.Tensor:
    if fmt == FMT_NVFP4:
        return F.mla_row_dequantize(pool)
    if fmt == FMT_FP8:
        return F.mla_fp8_row_dequantize(pool)
    raise ValueError(fmt)


def mla_decode_ref(q: torch.Tensor, pool: torch.Tensor, idx: torch.Tensor, sm_scale: float, fmt: int = FMT_NVFP4):
    """fp32 oracle: dequantizes only the referenced rows.  Returns (out [T, H, 512], lse [T, H]) on q's device."""
    dev = q.device
    qc, ic = q.float().cpu(), idx.cpu().long()
    used = torch.unique(ic[ic >= 0])
    if used.numel() == 0:
        t, h, _ = q.shape
        return (torch.zeros(t, h, F.MLA_NOPE, device=dev), torch.full((t, h), float("-inf"), device=dev))
    rows = dequant_rows(pool[used.to(pool.device)].cpu(), fmt)
    remap = torch.full((int(used.max()) + 1,), -1, dtype=torch.long)
    remap[used] = torch.arange(used.numel())
    table = torch.where(ic >= 0, remap[ic.clamp(min=0)], torch.full_like(ic, -1))
    o, l = F.sparse_mla_reference(qc, rows, table, sm_scale)
    return o.to(dev), l.to(dev)


def mla_sm_scale(qk_head_dim: int = 192) -> float:
    """DeepSeek-style softmax scale: 1 / sqrt(qk_nope_head_dim + qk_rope_head_dim) of the un-absorbed heads."""
    return 1.0 / math.sqrt(qk_head_dim)
