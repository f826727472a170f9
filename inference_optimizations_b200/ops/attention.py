"""GQA attention over the paged pool: split-K decode / speculative verify (csrc/attn_gqa_decode.cu) and the fp32
oracle.  Semantics of the reference's grouped decode and split-K verify (`attention/verify-splitk/gemma31_verify.py:1-24`,
`kv-cache-4bit/kv4tri-triton-backend/kv4tri_nvfp4_attention.py:257`): request b has kv_len[b] tokens in the pool, the
last n_q of which are its query tokens; query token t sees key positions p <= q_pos(t) and, with a sliding window W,
only q_pos(t) - p < W (W = 1024 on Gemma sliding layers: each query sees 1024 keys including itself).
Prefill chunks over NVFP4 / FP8 pools run the GQA-packed extend kernel (csrc/attn_gqa_extend.cu, `gqa_extend`): 128
query rows (128 / G tokens x G heads) per kv head and CTA, the reference's `attention/extend-gqa` capability."""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from .._ext import ext
from .kvcache import gqa_pool_read_ref

NUM_SMS = 148
TILE = 128


def split_policy(batch_heads: int, max_ctx: int, window: int = 0, target_ctas: int = 2 * NUM_SMS,
                 min_tiles: int = 4) -> tuple[int, int]:
    """(num_splits, tiles_per_split): enough CTAs to fill the 148 SMs twice, at least `min_tiles` 128-token tiles
    per split.  Fixed per (batch, context bound) so a captured CUDA graph keeps a valid schedule."""
    span = min(max_ctx, window + TILE) if window > 0 else max_ctx
    tiles = max(1, (span + TILE - 1) // TILE + (1 if window > 0 else 0))
    best, best_cost = 1, None
    overhead_tiles = 3.0          # per-CTA prologue / pipeline fill / epilogue, in tile units (measured timeline)
    for s in range(1, 17):
        if s > 1 and tiles // s < min_tiles:
            break
        ctas = batch_heads * s
        waves = -(-ctas // NUM_SMS)            # one CTA per SM at a time
        tps = -(-tiles // s)
        cost = waves * (tps + overhead_tiles) + (0.5 if s > 1 else 0.0)   # + split combine
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    tps = (tiles + best - 1) // best
    splits = (tiles + tps - 1) // tps
    return splits, tps


@dataclass
class DecodeWorkspace:
    o_part: torch.Tensor
    lse_part: torch.Tensor
    status: torch.Tensor

    @staticmethod
    def allocate(max_b: int, hk: int, max_splits: int, d: int, rmax: int = 16, device="cuda") -> "DecodeWorkspace":
        n = max_b * hk * max_splits * rmax
        return DecodeWorkspace(torch.empty(n * d, dtype=torch.float32, device=device),
                               torch.empty(n, dtype=torch.float32, device=device),
                               torch.zeros(1, dtype=torch.int32, device=device))


def gqa_decode(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor, kv_len: torch.Tensor, n_q: int,
               hk: int, fmt: int, sm_scale: float, window: int = 0, k_scale: float = 1.0, v_scale: float = 1.0,
               splits: Optional[tuple[int, int]] = None, ws: Optional[DecodeWorkspace] = None,
               max_ctx: Optional[int] = None, out: Optional[torch.Tensor] = None,
               req_idx: Optional[torch.Tensor] = None, trace: Optional[torch.Tensor] = None,
               exact: bool = False) -> torch.Tensor:
    """q bf16 [B * n_q, Hq, D] -> out bf16 [B * n_q, Hq, D].  Batch entry b uses page-table row req_idx[b]
    (default b).  NVFP4 / FP8 pools run E4M3 tensor-core operands unless `exact` (f16 operands, exact dequant);
    bf16 pools always run f16."""
    b = kv_len.shape[0]
    d = q.shape[-1]
    if out is None:
        out = torch.empty_like(q)
    if not q.is_cuda:
        pt = page_table if req_idx is None else page_table[req_idx.long()]
        out.copy_(gqa_decode_ref(q, pool, pt, kv_len, n_q, hk, fmt, sm_scale, window, k_scale, v_scale)
                  .to(out.dtype))
        return out
    if splits is None:
        if max_ctx is None:
            max_ctx = int(kv_len.max().item())
        splits = split_policy(b * hk, max_ctx, window)
    ns, tps = splits
    if ws is None:
        ws = DecodeWorkspace.allocate(b, hk, ns, d, device=q.device)
    ext().gqa_decode(q, pool, page_table, req_idx, kv_len, out, ws.o_part, ws.lse_part, ws.status, n_q, hk, 64, window, fmt,
                     tps, ns, sm_scale, k_scale, v_scale, trace, int(exact))
    return out


def gqa_decode_ref(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor, kv_len: torch.Tensor, n_q: int,
                   hk: int, fmt: int, sm_scale: float, window: int = 0, k_scale: float = 1.0,
                   v_scale: float = 1.0) -> torch.Tensor:
    b = kv_len.shape[0]
    hq, d = q.shape[1], q.shape[2]
    g = hq // hk
    out = torch.zeros(b * n_q, hq, d, dtype=torch.float32)
    for i in range(b):
        n = int(kv_len[i])
        k, v = gqa_pool_read_ref(pool, page_table[i].cpu(), n, fmt, d, k_scale, v_scale)   # [n, Hk, D]
        kk = k.repeat_interleave(g, dim=1)
        vv = v.repeat_interleave(g, dim=1)
        for t in range(n_q):
            qpos = n - n_q + t
            p = torch.arange(n)
            vis = p <= qpos
            if window > 0:
                vis &= (qpos - p) < window
            qi = q[i * n_q + t].float().cpu()                                  # [Hq, D]
            s = torch.einsum("hd,nhd->hn", qi, kk[vis]) * sm_scale
            pr = torch.softmax(s, dim=-1)
            out[i * n_q + t] = torch.einsum("hn,nhd->hd", pr, vv[vis])
    return out.to(q.device)


def extend_blocks(segments: list, g: int) -> list:
    """Extend-kernel work list for prefill segments [(first q row, tokens, position of the first token, page-table
    row)]: each segment is cut into blocks of 128 / G consecutive tokens (128 query rows of one kv head)."""
    bt = 128 // g
    out = []
    for r0, n, p0, row in segments:
        for o in range(0, n, bt):
            out.append((r0 + o, min(bt, n - o), p0 + o, row))
    return out


def gqa_extend(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor, blocks: torch.Tensor, hk: int,
               fmt: int, sm_scale: float, window: int = 0, k_scale: float = 1.0, v_scale: float = 1.0,
               out: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None,
               trace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Prefill attention of the query tokens listed in `blocks` (int32 [n, 4] from `extend_blocks`) over the paged
    NVFP4 / FP8 pool: q bf16 [rows, Hq, D] -> out [rows, Hq, D] (rows outside every block are left as they are).
    Row t of block (r0, n, p0, req) is the token at position p0 + t; it sees pool positions <= p0 + t (and > p0 + t -
    window).  E4M3 tensor-core operands (Q per-row scale, K, V, P), fp32 accumulation."""
    if out is None:
        out = torch.zeros_like(q)
    if not q.is_cuda:
        out.copy_(gqa_extend_ref(q, pool, page_table, blocks, hk, fmt, sm_scale, window, k_scale, v_scale, out))
        return out
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=q.device)
    ext().gqa_extend(q, pool, page_table, blocks, out, status, hk, window, fmt, sm_scale, k_scale, v_scale, trace)
    return out


def gqa_extend_ref(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor, blocks: torch.Tensor, hk: int,
                   fmt: int, sm_scale: float, window: int = 0, k_scale: float = 1.0, v_scale: float = 1.0,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 oracle of `gqa_extend` (dense attention over the dequantized pool)."""
    res = (out.float().cpu().clone() if out is not None else torch.zeros(q.shape, dtype=torch.float32))
    for r0, n, p0, row in blocks.tolist():
        kv_n = p0 + n
        k, v = gqa_pool_read_ref(pool, page_table[row].cpu(), kv_n, fmt, q.shape[2], k_scale, v_scale)
        res[r0:r0 + n] = dense_attention_ref(q[r0:r0 + n].cpu(), k, v, sm_scale, torch.arange(p0, p0 + n),
                                             torch.arange(kv_n), window)
    return res


def dense_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float, q_pos: torch.Tensor,
                        k_pos: torch.Tensor, window: int = 0) -> torch.Tensor:
    """fp32 GQA attention on contiguous tensors: q [Tq, Hq, D], k/v [Tk, Hk, D], causal by positions (+ window)."""
    hq, hk = q.shape[1], k.shape[1]
    g = hq // hk
    kk = k.float().repeat_interleave(g, dim=1)
    vv = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * sm_scale
    vis = k_pos[None, :] <= q_pos[:, None]
    if window > 0:
        vis &= (q_pos[:, None] - k_pos[None, :]) < window
    s = s.masked_fill(~vis[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.einsum("hqk,khd->qhd", p, vv)


def sm_scale_for(d: int) -> float:
    return 1.0 / math.sqrt(d)
