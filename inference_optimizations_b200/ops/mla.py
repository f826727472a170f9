"""Sparse MLA (DSA) decode over the compressed latent pool: csrc/attn_mla_decode.cu and its fp32 oracle.

Semantics of the reference's sparse FP4 decode (`kv-cache-4bit/glm-kv4/glm_kv4.py:575-622` `sparse_mla`, the native
`kv-cache-4bit/kv4mla/csrc/api.cpp:73` `sparse_decode`): query token t (H heads x 576 = 512 latent + 64 rope) attends to
the pool rows idx[t, :] (-1 = masked); K = the full row, V = its 512 latent values; returns out [T, H, 512] and the
natural-log LSE [T, H].  Rows are NVFP4 352-B rows (FMT_NVFP4), E4M3 576-B rows (FMT_FP8) or rope-free NVFP4
288-B rows (FMT_NVFP4_NOROPE, the GLM-Flash latent) or 320-B / 384-B DeepSeek V4 Pro cells (FMT_V4PRO, E4M3 rope;
FMT_V4PRO_BF16, bf16 rope); unquantized 1152-B bf16 rows (FMT_BF16) are the accuracy reference pool, attended by
the fp32 torch path on any device (no kernel reads them)."""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from .._ext import ext
from . import formats as F
from .kvcache import FMT_BF16, FMT_FP8, FMT_NVFP4

FMT_NVFP4_NOROPE = 3      # the rope-free 288-byte NVFP4 row (GLM-Flash latent): attention over the 512 latent dims
FMT_V4PRO = 4             # the 320-byte DeepSeek V4 Pro cell: 448 NVFP4 latent dims (dims 448..511 read as zero) + 64 E4M3
FMT_V4PRO_BF16 = 5        # the 384-byte V4 Pro cell: as FMT_V4PRO with 64 bf16 rope values (rounded to E4M3 for the QK MMA)
                          # rope; the output's dims 448..511 are zero
NUM_SMS = 148
TILE = 128                # rows per kernel tile (split granularity and lazy-rescale step)
ROW_BYTES = {FMT_NVFP4: F.MLA_ROW_BYTES, FMT_FP8: F.MLA_FP8_ROW_BYTES, FMT_NVFP4_NOROPE: F.GLMFLASH_ROW_BYTES,
             FMT_V4PRO: F.v4pro_cell_bytes("fp8"), FMT_V4PRO_BF16: F.v4pro_cell_bytes("bf16"),
             FMT_BF16: F.MLA_BF16_ROW_BYTES}


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
    q8: torch.Tensor           # E4M3 query, quantized per (token, head) by the kernel's first pass
    q_scale: torch.Tensor

    @staticmethod
    def allocate(tokens: int, heads: int, max_splits: int, device="cuda") -> "MlaWorkspace":
        n = max(1, tokens * heads * max_splits)
        return MlaWorkspace(torch.empty(n * 512, dtype=torch.float32, device=device),
                            torch.empty(n, dtype=torch.float32, device=device),
                            torch.zeros(1, dtype=torch.int32, device=device),
                            torch.empty(tokens, heads, 576, dtype=torch.uint8, device=device),
                            torch.empty(tokens, heads, dtype=torch.float32, device=device))

    def fits(self, tokens: int, heads: int, splits: int) -> bool:
        return (self.q8.shape[0] >= tokens and self.q8.shape[1] == heads
                and self.lse_part.numel() >= tokens * heads * splits)


def mla_decode(q: torch.Tensor, pool: torch.Tensor, idx: torch.Tensor, sm_scale: float, fmt: int = FMT_NVFP4,
               splits: Optional[tuple[int, int]] = None, ws: Optional[MlaWorkspace] = None,
               out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
               return_lse: bool = False, trace: Optional[torch.Tensor] = None, exact: bool = False):
    """q bf16 [T, H, 576], pool uint8 [rows, 352 | 576 | 1152], idx int32 [T, topk] -> out bf16 [T, H, 512]
    (and lse fp32 [T, H], natural log, with return_lse).  exact: fp32 attention over the exactly decoded rows
    (`mla_decode_exact`) instead of the kernel; bf16 rows always take it."""
    t, h, _ = q.shape
    if out is None:
        out = torch.empty(t, h, F.MLA_NOPE, dtype=torch.bfloat16, device=q.device)
    if return_lse and lse is None:
        lse = torch.empty(t, h, dtype=torch.float32, device=q.device)
    if not q.is_cuda or fmt == FMT_BF16 or exact:
        o, l = (mla_decode_exact(q, pool, idx, sm_scale, fmt) if fmt == FMT_BF16 or exact else
                mla_decode_ref(q, pool, idx, sm_scale, fmt))
        out.copy_(o.to(out.dtype))
        if lse is not None:
            lse.copy_(l)
        return (out, lse) if return_lse else out
    if splits is None:
        splits = mla_split_policy(t, idx.shape[1])
    ns, tps = splits
    if ws is None:
        ws = MlaWorkspace.allocate(t, h, ns, device=q.device)
    assert ws.fits(t, h, ns), "workspace too small"
    ext().mla_decode(q.contiguous(), ws.q8[:t], ws.q_scale[:t], pool, idx, out, lse, ws.o_part, ws.lse_part, ws.status,
                     fmt, tps, ns, sm_scale, trace, None, 0, 0)
    return (out, lse) if return_lse else out


def mla_decode_mixed(q: torch.Tensor, pools: list, fmts: list, row_los: list, idx: torch.Tensor,
                     tok_pool: torch.Tensor, sm_scale: float, ws: Optional[MlaWorkspace] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sparse MLA decode over a mixed-format page space (kvmix): pool k holds the rows [row_los[k], row_los[k] +
    rows_k) of one id space in format fmts[k]; every token's rows live in the pool tok_pool[t] names.  One launch per
    pool, each over all tokens, skipping those of the other pool (so a CUDA graph holds a fixed launch list whatever
    the requests' placement); the query is quantized once, by the first launch.  -> out bf16 [T, H, 512]."""
    t, h, _ = q.shape
    if out is None:
        out = torch.empty(t, h, F.MLA_NOPE, dtype=torch.bfloat16, device=q.device)
    if not q.is_cuda:
        sel = tok_pool.cpu()
        for k, (pool, fmt, lo) in enumerate(zip(pools, fmts, row_los)):
            rows = (sel == k).nonzero().flatten()
            if rows.numel():
                ik = idx[rows]
                ik = torch.where(ik >= 0, ik - lo, ik)
                o, _ = mla_decode_ref(q[rows], pool, ik, sm_scale, fmt)
                out[rows] = o.to(out.dtype)
        return out
    ns, tps = mla_split_policy(t, idx.shape[1])
    if ws is None:
        ws = MlaWorkspace.allocate(t, h, ns, device=q.device)
    assert ws.fits(t, h, ns), "workspace too small"
    for k, (pool, fmt, lo) in enumerate(zip(pools, fmts, row_los)):
        ext().mla_decode(q.contiguous() if k == 0 else None, ws.q8[:t], ws.q_scale[:t], pool, idx, out, None,
                         ws.o_part, ws.lse_part, ws.status, fmt, tps, ns, sm_scale, None, tok_pool, k, lo)
    return out


def dense_indices(page_table: torch.Tensor, kv_len: torch.Tensor, max_ctx: int, page: int = 64) -> torch.Tensor:
    """Dense MLA (every cached position attended, e.g. Kimi K2.7's MLA over a paged FP4 pool; the reference's dense
    mode of the same kernel, `kv-cache-4bit/kv4mla/csrc/api.cpp:167-257`): pool rows of positions [0, kv_len) from
    the page table, -1 past the length, padded to a multiple of 128 (the kernel's tile)."""
    t = kv_len.shape[0]
    width = max(TILE, -(-max_ctx // TILE) * TILE)
    pos = torch.arange(width, device=kv_len.device)
    pages = page_table[:, :(-(-width // page))].long()
    rows = pages.gather(1, (pos // page).expand(t, -1).clamp(max=pages.shape[1] - 1)) * page + pos % page
    return torch.where(pos[None, :] < kv_len[:, None], rows, torch.full_like(rows, -1)).int()


def mla_dense_decode(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor, kv_len: torch.Tensor,
                     sm_scale: float, fmt: int = FMT_NVFP4, max_ctx: Optional[int] = None, **kw):
    """Dense MLA decode over a paged latent pool (one query token per row of kv_len)."""
    if max_ctx is None:
        max_ctx = int(kv_len.max().item())
    return mla_decode(q, pool, dense_indices(page_table, kv_len, max_ctx), sm_scale, fmt, **kw)


def dequant_rows(pool: torch.Tensor, fmt: int) -> torch.Tensor:
    """Rows -> fp32 [rows, 576] (latent, rope); the rope-free row's rope part is zero."""
    if fmt == FMT_BF16:
        return pool.contiguous().view(torch.bfloat16).view(pool.shape[0], F.MLA_QK).float()
    if fmt == FMT_NVFP4:
        return F.mla_row_dequantize(pool)
    if fmt == FMT_FP8:
        return F.mla_fp8_row_dequantize(pool)
    if fmt == FMT_NVFP4_NOROPE:
        lat = F.glmflash_row_dequantize(pool)
        return torch.cat([lat, torch.zeros(lat.shape[0], 64, dtype=lat.dtype, device=lat.device)], -1)
    if fmt in (FMT_V4PRO, FMT_V4PRO_BF16):
        c = F.v4pro_cell_dequantize(pool, "fp8" if fmt == FMT_V4PRO else "bf16")                           # [rows, 448 latent + 64 rope]
        z = torch.zeros(c.shape[0], F.MLA_NOPE - F.V4P_NOPE, dtype=c.dtype, device=c.device)
        return torch.cat([c[:, :F.V4P_NOPE], z, c[:, F.V4P_NOPE:]], -1)
    raise ValueError(fmt)


def mla_decode_exact(q: torch.Tensor, pool: torch.Tensor, idx: torch.Tensor, sm_scale: float,
                     fmt: int = FMT_BF16, chunk: int = 32) -> tuple[torch.Tensor, torch.Tensor]:
    """Sparse MLA attention in fp32 on q's device over the rows `idx` selects, each decoded exactly from its pool
    format (unquantized bf16 rows, [rows, 1152] bytes, as they are), `chunk` tokens at a time (their rows gathered
    and decoded once per chunk).  The attention of the bf16 reference pool, and the exact-arithmetic arm of the
    accuracy gate for the quantized pools (the kernel also rounds the query to E4M3).  -> (out fp32 [T, H, 512],
    lse fp32 [T, H]; a token with no valid row gives 0 and -inf)."""
    t, h, _ = q.shape
    out = torch.zeros(t, h, F.MLA_NOPE, dtype=torch.float32, device=q.device)
    lse = torch.full((t, h), float("-inf"), dtype=torch.float32, device=q.device)
    for a in range(0, t, chunk):
        ic = idx[a:a + chunk].long()
        c, kk = ic.shape
        k = dequant_rows(pool[ic.clamp(min=0).flatten()], fmt).view(c, kk, F.MLA_QK)   # [c, topk, 576] fp32
        s = torch.einsum("chd,ckd->chk", q[a:a + chunk].float(), k) * sm_scale
        s = s.masked_fill((ic < 0)[:, None, :], float("-inf"))
        m = s.amax(-1, keepdim=True)
        ok = torch.isfinite(m)
        p = torch.where(ok, torch.exp(s - torch.where(ok, m, torch.zeros_like(m))), torch.zeros_like(s))
        den = p.sum(-1, keepdim=True)
        out[a:a + chunk] = torch.einsum("chk,ckd->chd", p / den.clamp(min=1e-30), k[..., :F.MLA_NOPE])
        lse[a:a + chunk] = torch.where(ok[..., 0], (m + torch.log(den.clamp(min=1e-30)))[..., 0],
                                       torch.full_like(m[..., 0], float("-inf")))
    return out, lse


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


def _e4m3(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float()


def mla_decode_emul_e4m3(q: torch.Tensor, pool: torch.Tensor, idx: torch.Tensor, sm_scale: float,
                         fmt: int = FMT_NVFP4, tiles_per_split: Optional[int] = None, tau: float = 8.0):
    """CPU emulation of the kernel's arithmetic: per-(token, head) E4M3 query, rows rounded to E4M3, 128-row tiles
    with the lazy running max (rescale only when a tile's max exceeds the reference by more than 2^tau),
    P = 2^(s - m) rounded to E4M3, the row sum over unrounded P; with `tiles_per_split`, each split runs that
    schedule on its own tiles and the partials merge by their base-2 LSE.  Agrees with the kernel up to fp32
    accumulation order; used to test the kernel tightly where the fp32 oracle can only bound the E4M3 error."""
    log2e = 1.4426950408889634
    qf = q.float().cpu()
    t, h, _ = qf.shape
    amax = qf.abs().amax(-1, keepdim=True)
    qs = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q8 = _e4m3(qf * (1.0 / qs))
    ic = idx.cpu().long()
    ntiles = -(-ic.shape[1] // TILE)
    tps = tiles_per_split or ntiles
    ninf = float("-inf")
    out = torch.zeros(t, h, F.MLA_NOPE)
    lse = torch.full((t, h), ninf)
    for i in range(t):
        parts = []
        for s0 in range(0, ntiles, tps):
            m = torch.full((h,), ninf)
            l = torch.zeros(h)
            o = torch.zeros(h, F.MLA_NOPE)
            for j in range(s0, min(ntiles, s0 + tps)):
                ids = ic[i, j * TILE:(j + 1) * TILE]
                valid = ids >= 0
                rows = torch.zeros(ids.numel(), F.MLA_QK)
                if valid.any():
                    rows[valid] = dequant_rows(pool[ids[valid].to(pool.device)].cpu(), fmt)
                k8 = _e4m3(rows)
                sc = (q8[i] @ k8.T) * (qs[i] * sm_scale * log2e)
                sc[:, ~valid] = ninf
                mt = sc.max(-1).values
                first = (m == ninf) & (mt > ninf)
                grow = (m > ninf) & (mt > m + tau)
                alpha = torch.where(grow, torch.exp2(m - mt), torch.ones_like(m))
                m = torch.where(first | grow, mt, m)
                l = l * alpha
                o = o * alpha[:, None]
                p = torch.where(sc == ninf, torch.zeros_like(sc), torch.exp2(sc - m[:, None]))
                l = l + p.sum(-1)
                o = o + _e4m3(p) @ k8[:, :F.MLA_NOPE]
            ok = l > 0
            on = torch.where(ok[:, None], o / l.clamp(min=1e-30)[:, None], torch.zeros_like(o))
            parts.append((on, torch.where(ok, m + torch.log2(l.clamp(min=1e-30)), torch.full_like(m, ninf))))
        lmax = torch.stack([p[1] for p in parts]).max(0).values
        num = torch.zeros(h, F.MLA_NOPE)
        den = torch.zeros(h)
        for on, l2 in parts:
            w = torch.where(l2 == ninf, torch.zeros_like(l2), torch.exp2(l2 - lmax))
            num += w[:, None] * on
            den += w
        ok = den > 0
        out[i] = torch.where(ok[:, None], num / den.clamp(min=1e-30)[:, None], torch.zeros_like(num))
        lse[i] = torch.where(ok, (lmax + torch.log2(den.clamp(min=1e-30))) / log2e, torch.full_like(den, ninf))
    return out.to(q.device), lse.to(q.device)


# ---------------------------------------------------------------------------------------------------------------
# The two MLA layouts a draft (or target) layer can run in -- the reference's MLA draft models keep both
# (`speculative/k3-mla-draft/k3_mla_draft/k3_mla_draft.py:1-25`: latent MQA 576/512 and expanded MHA padded to 256,
# equal to 1e-9): the absorbed form attends once over the shared latent rows (what the sparse-MLA decode kernel and
# the paged pools use); the expanded form decompresses per-head K = [c W_UK[h]^T ; k_pe] and V = c W_UV[h], zero-pads
# both to `pad` dims and runs ordinary multi-head attention (what a dense MHA kernel or a prefill GEMM path wants).
def mla_attention_latent(q_nope: torch.Tensor, q_pe: torch.Tensor, c_kv: torch.Tensor, k_pe: torch.Tensor,
                         w_uk: torch.Tensor, w_uv: torch.Tensor, sm_scale: float,
                         mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q_nope [T, H, dn], q_pe [T, H, dr], c_kv [S, L], k_pe [S, dr], w_uk [H, dn, L], w_uv [H, L, dv],
    mask [T, S] bool (True = visible) -> out [T, H, dv]."""
    q_lat = torch.einsum("thn,hnl->thl", q_nope, w_uk)
    s = (torch.einsum("thl,sl->ths", q_lat, c_kv) + torch.einsum("thr,sr->ths", q_pe, k_pe)) * sm_scale
    if mask is not None:
        s = s.masked_fill(~mask[:, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("thl,hlv->thv", torch.einsum("ths,sl->thl", p, c_kv), w_uv)


def mla_expand_kv(c_kv: torch.Tensor, k_pe: torch.Tensor, w_uk: torch.Tensor, w_uv: torch.Tensor,
                  pad: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """Latent rows -> per-head K [S, H, pad] ([nope ; rope ; 0]) and V [S, H, pad] ([v ; 0])."""
    s_, h, dn, dr, dv = c_kv.shape[0], w_uk.shape[0], w_uk.shape[1], k_pe.shape[1], w_uv.shape[2]
    assert dn + dr <= pad and dv <= pad
    k = torch.zeros(s_, h, pad, dtype=c_kv.dtype, device=c_kv.device)
    k[..., :dn] = torch.einsum("sl,hnl->shn", c_kv, w_uk)
    k[..., dn:dn + dr] = k_pe[:, None, :]
    v = torch.zeros(s_, h, pad, dtype=c_kv.dtype, device=c_kv.device)
    v[..., :dv] = torch.einsum("sl,hlv->shv", c_kv, w_uv)
    return k, v


def mla_attention_expanded(q_nope: torch.Tensor, q_pe: torch.Tensor, c_kv: torch.Tensor, k_pe: torch.Tensor,
                           w_uk: torch.Tensor, w_uv: torch.Tensor, sm_scale: float,
                           mask: Optional[torch.Tensor] = None, pad: int = 256) -> torch.Tensor:
    """The same attention as `mla_attention_latent` through the expanded MHA layout."""
    t, h, dn = q_nope.shape
    dr, dv = q_pe.shape[2], w_uv.shape[2]
    k, v = mla_expand_kv(c_kv, k_pe, w_uk, w_uv, pad)
    q = torch.zeros(t, h, pad, dtype=q_nope.dtype, device=q_nope.device)
    q[..., :dn] = q_nope
    q[..., dn:dn + dr] = q_pe
    s = torch.einsum("thd,shd->ths", q, k) * sm_scale
    if mask is not None:
        s = s.masked_fill(~mask[:, None, :], float("-inf"))
    return torch.einsum("ths,shd->thd", torch.softmax(s, dim=-1), v)[..., :dv]
