"""KV-cache writers and the GQA page layout (kernels in csrc/elementwise.cu).

GQA pool of one layer: uint8 [num_pages, Hk, 2 (K, V), part_bytes(fmt, D)], page = 64 tokens.
  part (bf16)  : 64 rows x 2D bytes
  part (fp8)   : 64 rows x D bytes                       E4M3 of x / scale (per-layer k_scale / v_scale)
  part (nvfp4) : 64 rows x D/2 code bytes, then 64 x D/16 E4M3 block scales  (x = e2m1 * block * global)
Row bytes are stored with their 16-byte chunks XOR-swizzled by the row index (`kv_swizzle_perm`), the layout the
decode kernel's shared-memory tiles want; the element encoding is the reference's NVFP4 / E4M3 one.
MLA pool: uint8 [slots, 352] (NVFP4 row) or [slots, 576] (FP8 row); indexer pool uint8 [slots, 132].
"""
from __future__ import annotations

from functools import lru_cache
from typing import Optional

import torch

from .._ext import ext
from . import formats as F
from .basic import apply_rope_ref

FMT_BF16, FMT_FP8, FMT_NVFP4 = 0, 1, 2
FMT_IDS = {"bf16": FMT_BF16, "fp8": FMT_FP8, "nvfp4": FMT_NVFP4}
PAGE = 64


def part_bytes(fmt: int, d: int, page: int = PAGE) -> int:
    if fmt == FMT_BF16:
        return page * d * 2
    if fmt == FMT_FP8:
        return page * d
    return page * (d // 2 + d // 16)


def row_bytes(fmt: int, d: int) -> int:
    return {FMT_BF16: 2 * d, FMT_FP8: d, FMT_NVFP4: d // 2}[fmt]


@lru_cache(maxsize=None)
def kv_swizzle_perm(row_bytes_: int, rows: int = PAGE) -> torch.Tensor:
    """int64 [rows, row_bytes]: physical byte position of logical byte b of row r (16-byte chunk XOR swizzle)."""
    nch = min(8, row_bytes_ // 16)
    b = torch.arange(row_bytes_)
    r = torch.arange(rows)[:, None]
    j = b >> 4
    pos = (j & ~(nch - 1)) | ((j ^ r) & (nch - 1))
    return (pos << 4) | (b & 15)


def _encode_rows(x: torch.Tensor, fmt: int, scale: float) -> tuple[torch.Tensor, Optional[torch.Tensor]]:
    """x fp32 [n, D] -> (row bytes uint8 [n, row_bytes] logical order, nvfp4 scales uint8 [n, D/16] or None)."""
    if fmt == FMT_BF16:
        return x.to(torch.bfloat16).view(torch.uint8).reshape(x.shape[0], -1), None
    if fmt == FMT_FP8:
        return (x / scale).to(torch.float8_e4m3fn).view(torch.uint8), None
    packed, s8 = F.nvfp4_quantize(x, scale)
    return packed, s8.view(torch.uint8)


def _decode_rows(rows: torch.Tensor, scales: Optional[torch.Tensor], fmt: int, scale: float, d: int) -> torch.Tensor:
    if fmt == FMT_BF16:
        return rows.contiguous().view(torch.bfloat16).float().reshape(rows.shape[0], d)
    if fmt == FMT_FP8:
        return rows.view(torch.float8_e4m3fn).float() * scale
    return F.nvfp4_dequantize(rows, scales.view(torch.float8_e4m3fn), scale)


def gqa_pool_write_ref(pool: torch.Tensor, slot: torch.Tensor, k: torch.Tensor, v: torch.Tensor, fmt: int,
                       k_scale: float = 1.0, v_scale: float = 1.0) -> None:
    """Oracle writer. k, v fp32 [T, Hk, D] (already bf16-rounded); slot [T] (-1 skipped)."""
    t_, hk, d = k.shape
    rb = row_bytes(fmt, d)
    perm = kv_swizzle_perm(rb)
    for part, (x, sc) in enumerate(((k, k_scale), (v, v_scale))):
        for t in range(t_):
            s = int(slot[t])
            if s < 0:
                continue
            page, off = divmod(s, PAGE)
            codes, scales = _encode_rows(x[t], fmt, sc)
            blk = pool[page, :, part]                                    # [Hk, part_bytes]
            row = torch.zeros(hk, rb, dtype=torch.uint8)
            row[:, perm[off]] = codes.cpu()
            blk[:, off * rb:(off + 1) * rb] = row.to(pool.device)
            if scales is not None:
                base = PAGE * rb
                blk[:, base + off * (d // 16): base + (off + 1) * (d // 16)] = scales


def gqa_pool_read_ref(pool: torch.Tensor, pages: torch.Tensor, n_tok: int, fmt: int, d: int,
                      k_scale: float = 1.0, v_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Oracle reader: logical tokens 0..n_tok-1 of one request (page list `pages`) -> K, V fp32 [n_tok, Hk, D]."""
    rb = row_bytes(fmt, d)
    perm = kv_swizzle_perm(rb)
    out = []
    for part, sc in ((0, k_scale), (1, v_scale)):
        toks = []
        for p in range((n_tok + PAGE - 1) // PAGE):
            blk = pool[int(pages[p]), :, part].cpu()                       # [Hk, part_bytes]
            n = min(PAGE, n_tok - p * PAGE)
            rows = blk[:, : PAGE * rb].reshape(-1, PAGE, rb)               # [Hk, 64, rb] physical
            logical = torch.gather(rows, 2, perm[None].expand_as(rows))    # undo the swizzle
            scales = blk[:, PAGE * rb: PAGE * rb + PAGE * (d // 16)].reshape(-1, PAGE, d // 16) \
                if fmt == FMT_NVFP4 else None
            hk = rows.shape[0]
            dec = _decode_rows(logical[:, :n].reshape(hk * n, rb),
                               scales[:, :n].reshape(hk * n, d // 16) if scales is not None else None, fmt, sc, d)
            toks.append(dec.reshape(hk, n, d).transpose(0, 1))
        out.append(torch.cat(toks, 0))
    return out[0], out[1]


def _head_rmsnorm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float, plus_one: bool) -> torch.Tensor:
    if w is None:
        return x
    inv = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    g = w.float() + 1.0 if plus_one else w.float()
    return (x * inv * g).to(torch.bfloat16).float()


def gqa_prep(qkv: torch.Tensor, q_norm: Optional[torch.Tensor], k_norm: Optional[torch.Tensor],
             cos_sin: torch.Tensor, pos: torch.Tensor, slot: torch.Tensor, pool: torch.Tensor, fmt: int,
             hq: int, hk: int, d: int, eps: float, plus_one: bool, k_scale: float = 1.0, v_scale: float = 1.0,
             q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused: per-head RMSNorm of q/k, NeoX RoPE, q -> bf16 [T, Hq, D], k/v -> pool[slot].  Returns q_out."""
    t = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty(t, hq, d, dtype=torch.bfloat16, device=qkv.device)
    if qkv.is_cuda:
        ext().gqa_prep(qkv, q_norm, k_norm, cos_sin, pos.int(), slot.int(), q_out, pool, fmt, k_scale, v_scale,
                       hq, hk, d, PAGE, eps, plus_one)
        return q_out
    x = qkv[:, : (hq + 2 * hk) * d].float().reshape(t, hq + 2 * hk, d)
    q = apply_rope_ref(_head_rmsnorm(x[:, :hq], q_norm, eps, plus_one), pos, cos_sin)
    k = apply_rope_ref(_head_rmsnorm(x[:, hq:hq + hk], k_norm, eps, plus_one), pos, cos_sin)
    v = x[:, hq + hk:]
    q_out.copy_(q.to(torch.bfloat16))
    gqa_pool_write_ref(pool, slot, k.to(torch.bfloat16).float(), v.to(torch.bfloat16).float(), fmt, k_scale, v_scale)
    return q_out


def mla_write(nope: torch.Tensor, rope: torch.Tensor, slot: torch.Tensor, pool: torch.Tensor) -> None:
    """Latent rows into an MLA pool ([slots, 352] NVFP4, [slots, 576] FP8 or [slots, 1152] unquantized bf16, the
    accuracy reference); slot -1 skipped."""
    if pool.shape[-1] == F.MLA_BF16_ROW_BYTES:
        rows = torch.cat([nope, rope], -1).to(torch.bfloat16).contiguous().view(torch.uint8)
        keep = slot >= 0
        pool[slot[keep].long()] = rows[keep]
        return
    fmt = FMT_NVFP4 if pool.shape[-1] == F.MLA_ROW_BYTES else FMT_FP8
    if nope.is_cuda:
        ext().mla_quant_write(nope, rope, slot.int(), pool, fmt)
        return
    rows = F.mla_row_quantize(nope, rope) if fmt == FMT_NVFP4 else F.mla_fp8_row_quantize(nope, rope)
    keep = slot >= 0
    pool[slot[keep].long()] = rows[keep]


# DSA indexer key pool: 132 bytes per token (128 E4M3 values + fp32 scale, `F.index_key_quantize`), stored per
# 64-token page as [64 x 128 B values][64 x fp32 scales] = 8448 B, the values of row r in the 128-byte-swizzle order
# (16-byte chunk c at c ^ (r & 7)).  A page is then a ready K-major tensor-core operand for one plain bulk copy.
INDEX_PAGE_BYTES = 64 * F.INDEX_ROW_BYTES


def index_pool_offsets(slot: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Byte offsets (values [n, 128], scale [n]) of the tokens in `slot` inside a flat index pool."""
    s = slot.long()
    page, r = s // 64, s % 64
    b = torch.arange(128, device=s.device)
    chunk = (b // 16)[None, :] ^ (r % 8)[:, None]
    vals = page[:, None] * INDEX_PAGE_BYTES + r[:, None] * 128 + chunk * 16 + (b % 16)[None, :]
    scale = page * INDEX_PAGE_BYTES + 64 * 128 + 4 * r
    return vals, scale


def index_key_write(k: torch.Tensor, slot: torch.Tensor, pool: torch.Tensor) -> None:
    """k [T, 128] -> pool [pages, 8448] uint8 at token slots (-1 = skip)."""
    if k.is_cuda:
        ext().index_key_write(k, slot.int(), pool)
        return
    keep = slot >= 0
    rows = F.index_key_quantize(k)[keep]
    vals, sc = index_pool_offsets(slot[keep])
    flat = pool.view(-1)
    flat[vals.reshape(-1)] = rows[:, :128].reshape(-1)
    sidx = sc[:, None] + torch.arange(4)[None, :]
    flat[sidx.reshape(-1)] = rows[:, 128:].reshape(-1)


def index_key_read(pool: torch.Tensor, slot: torch.Tensor) -> torch.Tensor:
    """Logical 132-byte rows [n, 132] of the tokens in `slot` (the inverse of index_key_write's layout)."""
    vals, sc = index_pool_offsets(slot)
    flat = pool.reshape(-1)
    sidx = sc[:, None] + torch.arange(4, device=pool.device)[None, :]
    return torch.cat([flat[vals], flat[sidx]], dim=1)
