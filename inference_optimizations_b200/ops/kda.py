"""Kimi Delta Attention (gated delta-rule linear attention) decode step and its recurrent-state storage formats.

`kda_decode` runs the fused CUDA kernel (csrc/kda.cu: conv -> gate -> L2 norm -> delta rule -> sigmoid-gated
RMSNorm in one launch per layer); `kda_decode_ref` is the fp32 oracle of the same math
(`linear-attention-kda/kda-fused-decode/kda.py:1-60` states the contract: value-major state, eps inside the root,
softplus threshold 20, SiLU conv, sigmoid output gate).

Recurrent-state rows (`kv-cache-4bit/k3-quantized-state/k3state_quant.py:1-37`): the state of one head is 128 value
rows of 128 fp32; a parked request's state is kept quantized per row -- FP8 (128 E4M3 + fp32 scale = 132 B),
bf16 (256 B) or NVFP4 (64 B E2M1 + 8 E4M3 block scales + fp32 global = 76 B) -- and expanded into an fp32 working
copy when the request runs again (`StateStore`).
"""
from __future__ import annotations

import torch
import torch.nn.functional as Fn

from .._ext import ext
from . import formats as F


def kda_decode_ref(q, k, v, g_proj, dt_bias, A_log, beta, g2, norm_w, cwq, cwk, cwv, csq, csk, csv, state,
                   scale=None):
    """Same arguments as `kda_decode` (states updated in place, fp32 math); returns o [B, HV, DV] bf16."""
    B, H, DK = q.shape
    HV, DV = v.shape[1], v.shape[2]
    W = cwq.shape[1]
    scale = DK ** -0.5 if scale is None else scale

    def conv(x, w, st):                      # x [B, C], w [C, W], st [B, C, W-1]
        y = (st * w[None, :, :W - 1]).sum(-1) + x * w[None, :, W - 1]
        st.copy_(torch.cat([st[..., 1:], x[..., None]], -1))
        return Fn.silu(y)

    qc = conv(q.float().reshape(B, -1), cwq, csq.view(B, H * DK, W - 1)).view(B, H, DK)
    kc = conv(k.float().reshape(B, -1), cwk, csk.view(B, H * DK, W - 1)).view(B, H, DK)
    vc = conv(v.float().reshape(B, -1), cwv, csv.view(B, HV * DV, W - 1)).view(B, HV, DV)
    gp = g_proj.float() + dt_bias.view(HV, DK)[None]
    sp = torch.where(gp > 20, gp, torch.log1p(torch.exp(gp)))
    g = -torch.exp(A_log.float())[None, :, None] * sp                     # [B, HV, DK], log-space decay
    rep = HV // H
    qn = qc / torch.sqrt((qc * qc).sum(-1, keepdim=True) + 1e-6) * scale
    kn = kc / torch.sqrt((kc * kc).sum(-1, keepdim=True) + 1e-6)
    qn, kn = qn.repeat_interleave(rep, 1), kn.repeat_interleave(rep, 1)
    h = state.view(B, HV, DV, DK)
    h.mul_(torch.exp(g)[:, :, None, :])
    err = vc - torch.einsum("bhvk,bhk->bhv", h, kn)
    bt = beta.float() if beta.dim() == 3 else beta.float()[..., None]
    u = err * bt
    h.add_(u[..., None] * kn[:, :, None, :])
    o = torch.einsum("bhvk,bhk->bhv", h, qn)
    o = o * torch.sigmoid(g2.float())
    o = o / torch.sqrt((o * o).mean(-1, keepdim=True) + 1e-5) * norm_w.float()
    return o.to(torch.bfloat16)


def kda_decode(q, k, v, g_proj, dt_bias, A_log, beta, g2, norm_w, cwq, cwk, cwv, csq, csk, csv, state, scale=None):
    """Fused decode step on the GPU (q/k heads == value heads, head dims 128); falls back to the oracle on CPU."""
    if not q.is_cuda:
        return kda_decode_ref(q, k, v, g_proj, dt_bias, A_log, beta, g2, norm_w, cwq, cwk, cwv, csq, csk, csv,
                              state, scale)
    out = torch.empty(v.shape, dtype=torch.bfloat16, device=v.device)
    ext().kda_decode(q, k, v, g_proj, dt_bias, A_log, beta, g2, norm_w, cwq, cwk, cwv, csq, csk, csv, state, out,
                     q.shape[2] ** -0.5 if scale is None else scale)
    return out


# ------------------------------------------------------------------------------------------------ chunked prefill
def kda_prefill(q, k, v, g_proj, dt_bias, A_log, beta, g2, norm_w, cwq, cwk, cwv, csq, csk, csv, state,
                scale=None, chunk: int = 64):
    """Prefill of T tokens per sequence in chunks (the FlashKDA idea, `linear-attention-kda/flashkda-split`: the
    sequential recurrence over T tokens becomes T / chunk sequential steps of dense chunk math).  Inputs are the
    decode step's with a time axis: q/k [B, T, H, DK], v [B, T, HV, DV], g_proj [B, T, HV, DK], beta [B, T, HV]
    (or [B, T, HV, DV]), g2 [B, T, HV, DV]; conv and recurrent states updated in place; returns o [B, T, HV, DV]
    bf16, equal to T calls of `kda_decode_ref` up to fp32 rounding.

    Within a chunk with state S0 (value-major [DV, DK]) and per-key-channel log decays G_t = cumsum(g) (so every
    exponent below is G_t - G_i <= 0): S_t = S0 diag(e^{G_t}) + sum_{i <= t} w_i (k_i * e^{G_t - G_i})^T, where the
    pseudo-values solve the unit-lower-triangular system
        w_t + beta_t * sum_{i < t} [(k_i * e^{G_t - G_i}) . k_t] w_i = beta_t * (v_t - S0 (k_t * e^{G_t}));
    then o_t = S_t q_t and S_C closes the chunk."""
    B, T, H, DK = q.shape
    HV, DV = v.shape[2], v.shape[3]
    W = cwq.shape[1]
    rep = HV // H
    scale = DK ** -0.5 if scale is None else scale

    def conv(x, w, st):                      # x [B, T, C], w [C, W], st [B, C, W-1]
        xx = torch.cat([st.transpose(1, 2), x], 1)                          # [B, T + W - 1, C]
        y = sum(xx[:, j:j + T] * w[None, None, :, j] for j in range(W))
        st.copy_(xx[:, T:].transpose(1, 2))
        return Fn.silu(y)

    qc = conv(q.float().reshape(B, T, -1), cwq, csq.view(B, H * DK, W - 1)).view(B, T, H, DK)
    kc = conv(k.float().reshape(B, T, -1), cwk, csk.view(B, H * DK, W - 1)).view(B, T, H, DK)
    vc = conv(v.float().reshape(B, T, -1), cwv, csv.view(B, HV * DV, W - 1)).view(B, T, HV, DV)
    gp = g_proj.float() + dt_bias.view(HV, DK)[None, None]
    sp = torch.where(gp > 20, gp, torch.log1p(torch.exp(gp)))
    g = -torch.exp(A_log.float())[None, None, :, None] * sp                 # [B, T, HV, DK]
    qn = (qc / torch.sqrt((qc * qc).sum(-1, keepdim=True) + 1e-6) * scale).repeat_interleave(rep, 2)
    kn = (kc / torch.sqrt((kc * kc).sum(-1, keepdim=True) + 1e-6)).repeat_interleave(rep, 2)
    bt = beta.float()
    # head-major [B, HV, T, .]
    qn, kn, vc, g = (t.transpose(1, 2) for t in (qn, kn, vc, g))
    bt = bt.transpose(1, 2)
    S = state.view(B, HV, DV, DK)
    out = torch.empty(B, HV, T, DV, dtype=torch.float32, device=q.device)
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        C = c1 - c0
        Kc, Qc, Vc = kn[:, :, c0:c1], qn[:, :, c0:c1], vc[:, :, c0:c1]
        G = torch.cumsum(g[:, :, c0:c1], 2)                                # [B, HV, C, DK]
        tri = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device))
        D = G[:, :, :, None, :] - G[:, :, None, :, :]                        # [B, HV, t, i, DK]
        E = torch.exp(D.masked_fill(~tri[None, None, :, :, None], float("-inf")))   # i <= t only (exponent <= 0)
        KK = torch.einsum("bhtd,bhid,bhtid->bhti", Kc, Kc, E)                # (k_i e^{G_t - G_i}) . k_t
        QK = torch.einsum("bhtd,bhid,bhtid->bhti", Qc, Kc, E)                # (k_i e^{G_t - G_i}) . q_t, i <= t
        strict = torch.tril(torch.ones(C, C, device=q.device), -1)
        Kt = Kc * torch.exp(G)                                               # k_t * e^{G_t}
        rhs = Vc - torch.einsum("bhtd,bhvd->bhtv", Kt, S)                   # v_t - S0 (k_t e^{G_t})
        if bt.dim() == 3:                                                    # one beta per head and token
            b_ = bt[:, :, c0:c1]
            A = torch.eye(C, device=q.device) + b_[..., None] * KK * strict
            Wv = torch.linalg.solve_triangular(A, b_[..., None] * rhs, upper=False, unitriangular=True)
        else:                                                                # a beta per value row
            b_ = bt[:, :, c0:c1].transpose(2, 3)                             # [B, HV, DV, C]
            A = torch.eye(C, device=q.device) + b_[..., None] * (KK * strict)[:, :, None]
            Wv = torch.linalg.solve_triangular(A, (b_ * rhs.transpose(2, 3))[..., None], upper=False,
                                               unitriangular=True)[..., 0].transpose(2, 3)
        out[:, :, c0:c1] = torch.einsum("bhtd,bhvd->bhtv", Qc * torch.exp(G), S) + torch.einsum(
            "bhti,bhiv->bhtv", QK, Wv)
        Gl = G[:, :, -1]                                                     # [B, HV, DK]
        S.mul_(torch.exp(Gl)[:, :, None, :]).add_(
            torch.einsum("bhiv,bhid->bhvd", Wv, Kc * torch.exp(Gl[:, :, None, :] - G)))
    o = out.transpose(1, 2) * torch.sigmoid(g2.float())                     # [B, T, HV, DV]
    o = o / torch.sqrt((o * o).mean(-1, keepdim=True) + 1e-5) * norm_w.float()
    return o.to(torch.bfloat16)


# ------------------------------------------------------------------------------------------------ state rows
ROW_BYTES = {"fp8": 132, "bf16": 256, "nvfp4": 76}


def quant_state_rows(rows: torch.Tensor, fmt: str) -> torch.Tensor:
    """fp32 [R, 128] -> uint8 [R, ROW_BYTES[fmt]]."""
    r = rows.float()
    n = r.shape[0]
    if fmt == "bf16":
        return r.to(torch.bfloat16).view(torch.uint8).reshape(n, 256)
    if fmt == "fp8":
        s = (r.abs().amax(-1, keepdim=True) / 448.0).clamp(min=1e-30)
        q = (r / s).to(torch.float8_e4m3fn).view(torch.uint8)
        return torch.cat([q, s.view(torch.uint8).reshape(n, 4)], -1)
    g = (r.abs().amax(-1) / (448.0 * 6.0)).clamp(min=1e-30)
    out = torch.empty(n, 76, dtype=torch.uint8, device=r.device)
    for i in range(n):                         # per-row global scale
        p, s8 = F.nvfp4_quantize(r[i:i + 1], float(g[i]))
        out[i, :64], out[i, 64:72] = p[0], s8[0].view(torch.uint8)
    out[:, 72:] = g.view(torch.uint8).reshape(n, 4)
    return out


def dequant_state_rows(b: torch.Tensor, fmt: str) -> torch.Tensor:
    n = b.shape[0]
    if fmt == "bf16":
        return b.contiguous().view(torch.bfloat16).float().reshape(n, 128)
    if fmt == "fp8":
        s = b[:, 128:].contiguous().view(torch.float32)
        return b[:, :128].contiguous().view(torch.float8_e4m3fn).float() * s
    g = b[:, 72:].contiguous().view(torch.float32)[:, 0]
    return torch.stack([F.nvfp4_dequantize(b[i, :64], b[i, 64:72].contiguous().view(torch.float8_e4m3fn),
                                           float(g[i])) for i in range(n)])


class StateStore:
    """Parked recurrent states kept as quantized rows; `load` expands a request's state into an fp32 working copy,
    `park` quantizes it back (the two-tier pool of the reference: fp32 working copy + quantized mirror)."""

    def __init__(self, fmt: str = "fp8"):
        self.fmt = fmt
        self.parked: dict = {}

    def park(self, rid, state: torch.Tensor) -> None:
        self.parked[rid] = (tuple(state.shape), quant_state_rows(state.reshape(-1, 128), self.fmt))

    def load(self, rid) -> torch.Tensor:
        shape, rows = self.parked.pop(rid)
        return dequant_state_rows(rows, self.fmt).reshape(shape)

    def nbytes(self) -> int:
        return sum(r.numel() for _, r in self.parked.values())


class KDASmallProjections:
    """The five small bf16 projections of a KDA layer: beta (b: H -> nb), the low-rank forget gate (f_a: H -> d,
    f_b: d -> P) and the low-rank output gate (g_a: H -> d, g_b: d -> P).

    Run separately they are five launch-bound GEMMs per layer.  `fuse()` packs them into one GEMM H -> nb + 2d
    (b | f_a | g_a) and one batched GEMM [2, M, d] x [2, d, P] (f_b, g_b), and re-points the five weights at views of
    the packed storage, so memory does not grow and the separate path stays valid
    (`linear-attention-kda/small-projection-fuse/kda_smallproj_fuse_hooks.py:1-40`).  Call `fuse()` before capturing
    a CUDA graph that reads the weights: it moves them."""

    def __init__(self, w_b: torch.Tensor, w_fa: torch.Tensor, w_fb: torch.Tensor, w_ga: torch.Tensor,
                 w_gb: torch.Tensor):
        h = w_b.shape[1]
        if not (w_fa.shape[1] == w_ga.shape[1] == h and w_fb.shape[1] == w_fa.shape[0] == w_ga.shape[0]
                == w_gb.shape[1] and w_fb.shape[0] == w_gb.shape[0]):
            raise ValueError("KDA small projections: shapes disagree")
        self.w_b, self.w_fa, self.w_fb, self.w_ga, self.w_gb = w_b, w_fa, w_fb, w_ga, w_gb
        self.w_a = None            # [nb + 2d, H] once fused
        self.w_lr = None           # [2, d, P] once fused

    def forward_separate(self, x: torch.Tensor) -> tuple:
        """x [M, H] -> (beta logits [M, nb], forget-gate projection [M, P], output-gate projection [M, P])."""
        b = Fn.linear(x, self.w_b)
        f = Fn.linear(Fn.linear(x, self.w_fa), self.w_fb)
        g = Fn.linear(Fn.linear(x, self.w_ga), self.w_gb)
        return b, f, g

    def fuse(self) -> None:
        if self.w_a is not None:
            return
        nb, d = self.w_b.shape[0], self.w_fa.shape[0]
        self.w_a = torch.cat([self.w_b, self.w_fa, self.w_ga], 0).contiguous()
        self.w_lr = torch.stack([self.w_fb.t(), self.w_gb.t()], 0).contiguous()          # [2, d, P]
        self.w_b, self.w_fa, self.w_ga = self.w_a[:nb], self.w_a[nb:nb + d], self.w_a[nb + d:]
        self.w_fb, self.w_gb = self.w_lr[0].t(), self.w_lr[1].t()

    def forward(self, x: torch.Tensor) -> tuple:
        if self.w_a is None:
            return self.forward_separate(x)
        nb, d = self.w_b.shape[0], self.w_fa.shape[0]
        a = Fn.linear(x, self.w_a)                                                       # [M, nb + 2d]
        lo = a[:, nb:].unflatten(1, (2, d)).transpose(0, 1)                              # [2, M, d]
        fg = torch.bmm(lo, self.w_lr)                                                    # [2, M, P]
        return a[:, :nb], fg[0], fg[1]
