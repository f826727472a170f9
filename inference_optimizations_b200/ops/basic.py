"""Normalisation, activation, embedding, sampling and RoPE-table ops (kernels in csrc/elementwise.cu)."""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._ext import ext


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, plus_one: bool = False,
            residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
            fp8: Optional[tuple] = None) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * (1 + w if plus_one else w).  With `residual`, first residual <- x + residual
    (in place, bf16) and normalise that sum (the fused add+norm of `attention/gemma-fused-glue/rtx_glue.py`).
    fp8 = (q8 uint8 [rows, H], qs int32 [rows, H / 128]): the CUDA kernel also writes y block-quantized for an FP8
    GEMM (E4M3 + UE8M0 per 128; the bytes of quantizing y afterwards)."""
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    if x.is_cuda:
        ext().rmsnorm(x, residual, out, weight, eps, plus_one, *(fp8 if fp8 is not None else (None, None)))
        return out
    xf = x.float()
    if residual is not None:
        xf = (xf + residual.float()).to(torch.bfloat16).float()
        residual.copy_(xf.to(residual.dtype))
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    g = weight.float() + 1.0 if plus_one else weight.float()
    out.copy_((xf * inv * g).to(out.dtype))
    return out


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def act_mul(gate_up: torch.Tensor, gelu: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[.., 2F] -> [.., F]: act(gate) * up with act = gelu_tanh (GeGLU) or silu (SwiGLU)."""
    f = gate_up.shape[-1] // 2
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], f, dtype=torch.bfloat16, device=gate_up.device)
    if gate_up.is_cuda:
        ext().act_mul(gate_up, out, gelu)
        return out
    g, u = gate_up.float()[..., :f], gate_up.float()[..., f:]
    a = gelu_tanh(g) if gelu else torch.nn.functional.silu(g)
    out.copy_((a * u).to(out.dtype))
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, scale: float = 1.0,
          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=torch.bfloat16, device=table.device)
    if table.is_cuda:
        ext().embed(ids.int(), table, out, scale)
        return out
    e = table[ids.long()].float()
    out.copy_((e * scale).to(torch.bfloat16) if scale != 1.0 else e.to(torch.bfloat16))
    return out


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None,
           val: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row argmax (smallest index on ties) -> int32 [rows]."""
    rows = logits.numel() // logits.shape[-1]
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        ext().argmax(logits, out, val)
        return out
    lf = logits.float().reshape(rows, -1)
    m = lf.max(dim=-1, keepdim=True).values
    idx = torch.where(lf == m, torch.arange(lf.shape[1]).expand_as(lf), lf.shape[1]).min(dim=-1).values
    out.copy_(idx.to(torch.int32))
    if val is not None:
        val.copy_(m.squeeze(-1))
    return out


def rope_table(max_pos: int, dim: int, theta: float, device=None) -> torch.Tensor:
    """fp32 [max_pos, dim]: cos(p * theta^(-2i/dim)) for i < dim/2, then the sines (NeoX rotate-half RoPE).
    Angles are computed in float64 so long positions keep full fp32 accuracy."""
    half = dim // 2
    inv = theta ** (-torch.arange(half, dtype=torch.float64) * 2.0 / dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1).to(torch.float32).to(device)


def apply_rope_ref(x: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, D] fp32, NeoX rotate-half."""
    d = x.shape[-1]
    cs = cos_sin[pos.long()]
    c, s = cs[:, None, : d // 2], cs[:, None, d // 2:]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
