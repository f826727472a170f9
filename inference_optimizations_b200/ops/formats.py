"""KV-cache and activation number formats, with fp32 torch oracles (CPU or GPU) that the CUDA kernels must match.

Formats kept byte-compatible with the reference (the encoding is a contract between writer and reader kernels):

* NVFP4 MLA row, 352 bytes per token and layer (`kv-cache-4bit/glm-kv4/glm_kv4.py:1-36`):
    [0, 256)   512 E2M1 codes of the latent, element 2i in the low nibble of byte i
    [256, 288) one E4M3 scale per 16 latent values
    [288, 352) the 64 rope values as E4M3
  Per block of 16: scale = e4m3(clamp(amax / 6, 2^-9, 448)); code = E2M1(|x| / scale) where a value exactly on a
  midpoint (0.25 0.75 1.25 1.75 2.5 3.5 5) rounds DOWN and anything above 6 saturates; the sign bit (bit 3) is set
  only for a nonzero magnitude, so code 8 (-0) never appears.
* FP8 MLA row, 576 bytes: 512 E4M3 latent + 64 E4M3 rope (the row the FP8 baseline reads).
* NVFP4 per-head KV for GQA pools (`kv-cache-4bit/kv4tri-triton-backend/kv4tri_nvfp4_attention.py:9-14`): per head
  vector of D values, D/2 bytes of E2M1 pairs (same nibble order) + D/16 E4M3 block scales, times a per-layer fp32
  global scale: x = e2m1 * block_scale * global_scale.  The block scale uses the MLA rule on x / global_scale.
  The page-major arrangement of these bytes in the pool is this framework's own (see `kv/pool.py`).
* DSA indexer key, 132 bytes: 128 E4M3 values + one fp32 scale (`tooling/rooflines/glm_roofline.py:43-50`).
* FP8 activation quant with per-128 power-of-two (UE8M0) scales (`moe-gemm/norm-quant-fused/pro_norm_quant.py:1-17`):
  e = ceil(log2(amax / 448)), scale = 2^e, q = e4m3(x / scale).
* Rope-free NVFP4 row, 288 bytes (GLM-Flash DSA layers, kv_lora 512 and no rope; `kv-cache-4bit/glmflash-kv4/
  glmflash_kv4.py:1-20`): the first 288 bytes of the 352-byte row, same encoding.
* DeepSeek V4 Pro 4-bit cell, 320 bytes (rope E4M3) or 384 bytes (rope bf16) (`kv-cache-4bit/kv4pro-deepseek/
  kv4pro_fp4.py:1-30`): [0, 224) 448 nope values as E2M1 pairs, [224, 252) 28 E4M3 scales (one per 16), [252, 256)
  zero, [256, ..) rope.  Per 16-block the scale is e4m3(min(amax / 6 * f, 448)) for the f in (1, 0.93, 0.86, 0.8)
  with the smallest squared error, q = x * (1 / scale), E2M1 rounding to nearest with ties to even (unlike the MLA
  row's ties-down) and saturation at 6.
"""
from __future__ import annotations

import torch

MLA_NOPE = 512
MLA_ROPE = 64
MLA_QK = MLA_NOPE + MLA_ROPE          # 576
FP4_BLOCK = 16
MLA_SCALE_OFF = MLA_NOPE // 2         # 256
MLA_ROPE_OFF = MLA_SCALE_OFF + MLA_NOPE // FP4_BLOCK   # 288
MLA_ROW_BYTES = MLA_ROPE_OFF + MLA_ROPE                # 352
MLA_FP8_ROW_BYTES = MLA_QK                             # 576
MLA_BF16_ROW_BYTES = 2 * MLA_QK                        # 1152: unquantized bf16 row (the accuracy reference pool)
INDEX_DIM = 128
INDEX_ROW_BYTES = INDEX_DIM + 4                        # 132

E2M1_MAX = 6.0
E4M3_MAX = 448.0
SCALE_FLOOR = 2.0 ** -9               # smallest positive E4M3 (subnormal)

_E2M1_MAG = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_E2M1_EDGES = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def e2m1_table(device=None) -> torch.Tensor:
    """fp32 [16]: value of each 4-bit code (bit 3 = sign)."""
    mag = torch.tensor(_E2M1_MAG, dtype=torch.float32, device=device)
    return torch.cat([mag, -mag])


def e2m1_encode(y: torch.Tensor) -> torch.Tensor:
    """Signed fp32 values already divided by their block scale -> int32 codes 0..15 (ties down, saturating, no -0)."""
    edges = torch.tensor(_E2M1_EDGES, dtype=torch.float32, device=y.device)
    mag = torch.bucketize(y.abs().clamp(max=E2M1_MAX).contiguous(), edges, right=False).to(torch.int32)
    neg = (y < 0) & (mag > 0)
    return mag | (neg.to(torch.int32) << 3)


def e2m1_decode(codes: torch.Tensor) -> torch.Tensor:
    return e2m1_table(codes.device)[codes.long()]


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """int codes [..., 2n] -> uint8 [..., n]: element 2i low nibble, 2i+1 high nibble."""
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).to(torch.uint8)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    p = packed.to(torch.int32)
    return torch.stack([p & 0xF, p >> 4], dim=-1).flatten(-2)


def block_scale_e4m3(amax: torch.Tensor) -> torch.Tensor:
    """fp32 amax per 16-block -> E4M3 scale (as float8_e4m3fn)."""
    return (amax / E2M1_MAX).clamp(min=SCALE_FLOOR, max=E4M3_MAX).to(torch.float8_e4m3fn)


def nvfp4_quantize(x: torch.Tensor, global_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """x [..., D] (D % 16 == 0) -> (packed uint8 [..., D/2], scales float8_e4m3fn [..., D/16])."""
    d = x.shape[-1]
    xb = (x.float() / global_scale).reshape(*x.shape[:-1], d // FP4_BLOCK, FP4_BLOCK)
    s8 = block_scale_e4m3(xb.abs().amax(dim=-1))
    sf = s8.float()
    y = xb / sf.unsqueeze(-1)
    codes = e2m1_encode(y).reshape(*x.shape[:-1], d)
    return pack_nibbles(codes), s8


def nvfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor, global_scale: float = 1.0) -> torch.Tensor:
    """Inverse of nvfp4_quantize -> fp32 [..., D] (exact: value(code) * scale * global)."""
    vals = e2m1_decode(unpack_nibbles(packed))
    d = vals.shape[-1]
    vals = vals.reshape(*vals.shape[:-1], d // FP4_BLOCK, FP4_BLOCK) * scales.float().unsqueeze(-1)
    return vals.reshape(*vals.shape[:-2], d) * global_scale


# ------------------------------------------------------------------------------------------------ MLA rows


def mla_row_quantize(nope: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
    """nope [T, 512], rope [T, 64] (any float dtype) -> uint8 [T, 352] NVFP4 rows."""
    t = nope.shape[0]
    packed, s8 = nvfp4_quantize(nope)
    out = torch.empty(t, MLA_ROW_BYTES, dtype=torch.uint8, device=nope.device)
    out[:, :MLA_SCALE_OFF] = packed
    out[:, MLA_SCALE_OFF:MLA_ROPE_OFF] = s8.view(torch.uint8)
    out[:, MLA_ROPE_OFF:] = rope.float().to(torch.float8_e4m3fn).view(torch.uint8)
    return out


def mla_row_dequantize(rows: torch.Tensor) -> torch.Tensor:
    """uint8 [R, 352] -> fp32 [R, 576]."""
    nope = nvfp4_dequantize(rows[:, :MLA_SCALE_OFF], rows[:, MLA_SCALE_OFF:MLA_ROPE_OFF].view(torch.float8_e4m3fn))
    rope = rows[:, MLA_ROPE_OFF:].view(torch.float8_e4m3fn).float()
    return torch.cat([nope, rope], dim=-1)


def mla_fp8_row_quantize(nope: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
    """nope [T, 512], rope [T, 64] -> uint8 [T, 576] (E4M3, unit scale)."""
    return torch.cat([nope.float(), rope.float()], dim=-1).to(torch.float8_e4m3fn).view(torch.uint8)


def mla_fp8_row_dequantize(rows: torch.Tensor) -> torch.Tensor:
    return rows.view(torch.float8_e4m3fn).float()


def sparse_mla_reference(q: torch.Tensor, kv: torch.Tensor, table: torch.Tensor, sm_scale: float,
                         v_dim: int = MLA_NOPE) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 sparse MLA attention. q [T, H, 576], kv fp32 [N, 576] (dequantized pool), table [T, K] slots with -1
    masked. Returns (out [T, H, v_dim], lse [T, H] natural log; rows with no valid slot give 0 and -inf)."""
    t, h, _ = q.shape
    out = torch.zeros(t, h, v_dim, dtype=torch.float32, device=q.device)
    lse = torch.full((t, h), float("-inf"), dtype=torch.float32, device=q.device)
    for i in range(t):
        idx = table[i].long()
        idx = idx[idx >= 0]
        if idx.numel() == 0:
            continue
        k = kv[idx]
        s = (q[i].float() @ k.T) * sm_scale
        lse[i] = torch.logsumexp(s, dim=-1)
        out[i] = torch.softmax(s, dim=-1) @ k[:, :v_dim]
    return out, lse


# ------------------------------------------------------------------------------------------------ activations


GLMFLASH_ROW_BYTES = MLA_ROPE_OFF                      # 288


def glmflash_row_quantize(nope: torch.Tensor) -> torch.Tensor:
    """nope [T, 512] -> uint8 [T, 288] rope-free NVFP4 rows."""
    q, s8 = nvfp4_quantize(nope.float())
    return torch.cat([q, s8.view(torch.uint8)], dim=-1)


def glmflash_row_dequantize(rows: torch.Tensor) -> torch.Tensor:
    return nvfp4_dequantize(rows[:, :MLA_SCALE_OFF], rows[:, MLA_SCALE_OFF:GLMFLASH_ROW_BYTES].contiguous().view(
        torch.float8_e4m3fn))


V4P_NOPE, V4P_ROPE = 448, 64
V4P_SCALE_OFF, V4P_ROPE_OFF = 224, 256
V4P_SCALE_SEARCH = (1.0, 0.93, 0.86, 0.8)
_E2M1_EVEN = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)       # > at 0.25 / 1.25 / 2.5 / 5, >= at 0.75 / 1.75 / 3.5


def v4pro_cell_bytes(rope: str = "fp8") -> int:
    return V4P_ROPE_OFF + (V4P_ROPE if rope == "fp8" else 2 * V4P_ROPE)


def _e2m1_mag_even(a: torch.Tensor) -> torch.Tensor:
    a = a.clamp(max=E2M1_MAX)
    return ((a > 0.25).int() + (a >= 0.75).int() + (a > 1.25).int() + (a >= 1.75).int() + (a > 2.5).int()
            + (a >= 3.5).int() + (a > 5.0).int())


def v4pro_cell_quantize(x: torch.Tensor, rope: str = "fp8") -> torch.Tensor:
    """x [N, 512] (448 nope + 64 rope) -> uint8 [N, 320 | 384] cells (scale search, ties-to-even E2M1).  The block
    error is summed sequentially over the 16 values (the writer kernel's order)."""
    x = x.float()
    n = x.shape[0]
    nope = x[:, :V4P_NOPE].reshape(n, V4P_NOPE // FP4_BLOCK, FP4_BLOCK)
    amax = nope.abs().amax(-1)
    table = torch.tensor(_E2M1_MAG, device=x.device)
    best = None
    for f in V4P_SCALE_SEARCH:
        s8 = ((amax / E2M1_MAX) * torch.tensor(f, dtype=torch.float32)).clamp(max=E4M3_MAX).to(torch.float8_e4m3fn)
        sf = s8.float()
        inv = torch.where(sf > 0, 1.0 / torch.where(sf > 0, sf, torch.ones_like(sf)), torch.zeros_like(sf))
        q = nope * inv[..., None]
        mag = _e2m1_mag_even(q.abs())
        code = mag | (((q < 0) & (mag > 0)).int() << 3)
        d = torch.where(q < 0, -table[mag], table[mag]) * sf[..., None] - nope
        err = torch.zeros_like(amax)
        for j in range(FP4_BLOCK):
            err = err + d[..., j] * d[..., j]
        if best is None:
            best = [code, s8.view(torch.uint8), err]
        else:
            m = err < best[2]
            best = [torch.where(m[..., None], code, best[0]), torch.where(m, s8.view(torch.uint8), best[1]),
                    torch.where(m, err, best[2])]
    code = best[0].reshape(n, V4P_NOPE)
    cells = torch.zeros(n, v4pro_cell_bytes(rope), dtype=torch.uint8, device=x.device)
    cells[:, :V4P_SCALE_OFF] = pack_nibbles(code)
    cells[:, V4P_SCALE_OFF:V4P_SCALE_OFF + V4P_NOPE // FP4_BLOCK] = best[1]
    r = x[:, V4P_NOPE:]
    if rope == "fp8":
        cells[:, V4P_ROPE_OFF:] = r.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        cells[:, V4P_ROPE_OFF:] = r.to(torch.bfloat16).contiguous().view(torch.uint8)
    return cells


def v4pro_cell_dequantize(cells: torch.Tensor, rope: str = "fp8") -> torch.Tensor:
    """uint8 [N, 320 | 384] -> fp32 [N, 512]."""
    n = cells.shape[0]
    vals = e2m1_decode(unpack_nibbles(cells[:, :V4P_SCALE_OFF]))
    sf = cells[:, V4P_SCALE_OFF:V4P_SCALE_OFF + V4P_NOPE // FP4_BLOCK].contiguous().view(torch.float8_e4m3fn).float()
    nope = (vals.reshape(n, -1, FP4_BLOCK) * sf[..., None]).reshape(n, V4P_NOPE)
    if rope == "fp8":
        r = cells[:, V4P_ROPE_OFF:V4P_ROPE_OFF + V4P_ROPE].contiguous().view(torch.float8_e4m3fn).float()
    else:
        r = cells[:, V4P_ROPE_OFF:V4P_ROPE_OFF + 2 * V4P_ROPE].contiguous().view(torch.bfloat16).float()
    return torch.cat([nope, r], 1)


def fp8_quant_ue8m0(x: torch.Tensor, group: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """x [M, K] -> (q float8_e4m3fn [M, K], scale fp32 [M, K/group] powers of two). scale = 2^ceil(log2(amax/448))."""
    m, k = x.shape
    xg = x.float().reshape(m, k // group, group)
    amax = xg.abs().amax(dim=-1).clamp(min=1e-10)
    e = torch.ceil(torch.log2(amax / E4M3_MAX))
    s = torch.exp2(e)
    q = (xg / s.unsqueeze(-1)).to(torch.float8_e4m3fn).reshape(m, k)
    return q, s


def fp8_quant_block(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Weight [N, K] -> (q float8_e4m3fn [N, K], scale fp32 [N/128, K/128]) with scale = amax/448 per 128x128 block."""
    n, k = w.shape
    wb = w.float().reshape(n // block, block, k // block, block)
    amax = wb.abs().amax(dim=(1, 3)).clamp(min=1e-10)
    s = amax / E4M3_MAX
    q = (wb / s[:, None, :, None]).to(torch.float8_e4m3fn).reshape(n, k)
    return q, s


def fp8_dequant_block(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    n, k = q.shape
    return (q.float().reshape(n // block, block, k // block, block) * s[:, None, :, None]).reshape(n, k)


def index_key_quantize(k: torch.Tensor) -> torch.Tensor:
    """Indexer keys [T, 128] -> uint8 [T, 132]: E4M3 values scaled by amax/448, then the fp32 scale."""
    t = k.shape[0]
    amax = k.float().abs().amax(dim=-1, keepdim=True).clamp(min=1e-10)
    s = amax / E4M3_MAX
    q = (k.float() / s).to(torch.float8_e4m3fn).view(torch.uint8)
    return torch.cat([q, s.view(torch.uint8).reshape(t, 4)], dim=-1)


def index_key_dequantize(rows: torch.Tensor) -> torch.Tensor:
    q = rows[:, :INDEX_DIM].view(torch.float8_e4m3fn).float()
    s = rows[:, INDEX_DIM:].contiguous().view(torch.float32)
    return q * s
