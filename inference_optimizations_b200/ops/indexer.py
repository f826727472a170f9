"""DSA lightning indexer: relevance scores over the cached positions and the top-k positions per query token
(csrc/indexer.cu), with fp32 oracles.

score[t, j] = k_scale[j] * sum_h w[t, h] * relu(q[t, h] . k[j]) for j < limit[t] (the reference's indexer
semantics, `negative-results/code/idx_epilogue/triton_mla_logits.py:1-12`); top-k keeps the `topk` best positions
(lower position first on ties), returned in ascending position order as pool slots (page_table) and positions,
padded with -1 (`upstream-fixes/hooks/kpool_logits_chunk_hooks.py` row-wise top-2048 with -1 padding)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .._ext import ext
from . import formats as F
from .kvcache import index_key_read

TILE = 128


def indexer_q_quant(q: torch.Tensor, weights: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """q [T, Hi, 128] (any float), weights [T, Hi] -> (E4M3 q as uint8 [T, Hi, 128], w_eff [T, Hi] fp32 with the
    per-(token, head) query scale folded in: relu(s * x) = s * relu(x) for s > 0)."""
    qf = q.float()
    amax = qf.abs().amax(-1, keepdim=True)
    s = torch.where(amax > 0, amax / F.E4M3_MAX, torch.ones_like(amax))
    q8 = (qf / s).clamp(-F.E4M3_MAX, F.E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    return q8.contiguous(), (weights.float() * s[..., 0]).contiguous()


def indexer_scores_ref(q8: torch.Tensor, w: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor,
                       limit: torch.Tensor, width: int, req_idx: Optional[torch.Tensor] = None) -> torch.Tensor:
    t = q8.shape[0]
    out = torch.full((t, width), float("-inf"))
    qf = q8.cpu().view(torch.float8_e4m3fn).float()
    pt = page_table.cpu().long()
    for i in range(t):
        n = int(limit[i])
        if n == 0:
            continue
        row = int(req_idx[i]) if req_idx is not None else i
        pos = torch.arange(n)
        slot = pt[row][pos // 64] * 64 + pos % 64
        keys = index_key_read(pool.cpu(), slot)
        kv = keys[:, :128].contiguous().view(torch.float8_e4m3fn).float()
        ks = keys[:, 128:].contiguous().view(torch.float32)[:, 0]
        logits = torch.relu(qf[i] @ kv.T)                              # [Hi, n]
        out[i, :n] = ks * (w[i].float().cpu() @ logits)
    return out


def topk_ref(scores: torch.Tensor, limit: torch.Tensor, topk: int, page_table: torch.Tensor,
             req_idx: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Positions of the topk largest scores per row (ties -> lower position), ascending, -1 padded; and slots."""
    t = scores.shape[0]
    pos_out = torch.full((t, topk), -1, dtype=torch.int32)
    slot_out = torch.full((t, topk), -1, dtype=torch.int32)
    pt = page_table.cpu().long()
    for i in range(t):
        n = min(int(limit[i]), scores.shape[1])
        if n <= topk:
            sel = torch.arange(n)
        else:
            s = scores[i, :n].cpu()
            order = sorted(range(n), key=lambda j: (-float(s[j]), j))[:topk]
            sel = torch.tensor(sorted(order))
        row = int(req_idx[i]) if req_idx is not None else i
        pos_out[i, :len(sel)] = sel.int()
        slot_out[i, :len(sel)] = (pt[row][sel // 64] * 64 + sel % 64).int()
    return slot_out, pos_out


@dataclass
class IndexerWorkspace:
    scores: torch.Tensor
    status: torch.Tensor

    @staticmethod
    def allocate(tokens: int, max_ctx: int, device="cuda") -> "IndexerWorkspace":
        width = max(TILE, -(-max_ctx // TILE) * TILE)
        return IndexerWorkspace(torch.empty(tokens, width, dtype=torch.float32, device=device),
                                torch.zeros(1, dtype=torch.int32, device=device))


# fp32 score rows one selection call may hold (tokens x context x 4 B): a long prefill chunk over a long context
# (8192 tokens x 204,800 positions = 6.7 GB) selects in row blocks under this instead
SCORE_BYTES_MAX = 1 << 30


def indexer_select(q8: torch.Tensor, w: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor,
                   limit: torch.Tensor, topk: int, max_ctx: int, req_idx: Optional[torch.Tensor] = None,
                   ws: Optional[IndexerWorkspace] = None, tiles_per_cta: int = 0,
                   with_pos: bool = False):
    """-> slots int32 [T, topk] (and positions with `with_pos`).  `max_ctx` bounds limit (fixed per CUDA graph).
    tiles_per_cta 0: as many 128-position tiles per CTA as fill every SM about once (at most 32), so a decode step
    of a few tokens still spreads its score pass over the GPU; depends only on (T, max_ctx), so graphs stay valid.
    Without a workspace, a step whose score rows exceed SCORE_BYTES_MAX runs in blocks of rows (exact: a token's
    selection reads only its own row)."""
    t = q8.shape[0]
    width = max(TILE, -(-max_ctx // TILE) * TILE)
    block = max(1, SCORE_BYTES_MAX // (4 * width))
    if ws is None and t > block:
        rix = req_idx if req_idx is not None else torch.arange(t, dtype=torch.int32, device=q8.device)
        parts = [indexer_select(q8[a:a + block], w[a:a + block], pool, page_table, limit[a:a + block], topk,
                                max_ctx, rix[a:a + block], None, tiles_per_cta, with_pos)
                 for a in range(0, t, block)]
        if with_pos:
            return torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])
        return torch.cat(parts)
    slots = torch.empty(t, topk, dtype=torch.int32, device=q8.device)
    pos = torch.empty(t, topk, dtype=torch.int32, device=q8.device) if with_pos else None
    if not q8.is_cuda:
        sc = indexer_scores_ref(q8, w, pool, page_table, limit, max_ctx, req_idx)
        s_, p_ = topk_ref(sc, limit, topk, page_table, req_idx)
        slots.copy_(s_)
        if pos is not None:
            pos.copy_(p_)
        return (slots, pos) if with_pos else slots
    if ws is None:
        ws = IndexerWorkspace.allocate(t, max_ctx, q8.device)
    max_tiles = max(1, -(-max_ctx // TILE))
    if tiles_per_cta <= 0:
        tiles_per_cta = max(1, min(32, -(-t * max_tiles // 148)))
    ext().indexer(q8, w, pool, page_table, req_idx, limit, ws.scores, slots, pos, ws.status,
                  min(tiles_per_cta, max_tiles), max_tiles, 1, 1)
    return (slots, pos) if with_pos else slots
