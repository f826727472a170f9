"""Routed mixture of experts (DeepSeek-V3 class): sigmoid router with bias-corrected, group-limited top-k selection,
SwiGLU experts, shared expert.

Router semantics (the `noaux_tc` router the reference serves; `moe-gemm/router-piggyback/dp_router_piggyback.py:1-25`
carries its top-k ids / weights): scores = sigmoid(x W_gate^T); selection uses scores + e_bias; with n_group > 1 the
experts are split into groups, a group's score is the sum of its two best biased scores, only the topk_group best
groups stay eligible; the top-k experts' *unbiased* scores are renormalised to sum 1 and scaled by routed_scale.
`router="softmax"`: softmax over experts, top-k, renormalised (Qwen / Mixtral style).
"""
from __future__ import annotations

import torch
import torch.nn.functional as Fn

from .._ext import ext


def route(logits: torch.Tensor, e_bias: torch.Tensor, topk: int, n_group: int, topk_group: int,
          routed_scale: float, kind: str = "sigmoid", ksplit: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """logits fp32 [T, E] -> (expert ids int32 [T, topk], weights fp32 [T, topk]).  Ties: lower expert id.
    ksplit > 1 (CUDA, E and E / n_group multiples of 32): `logits` is the router GEMM's split-K partials
    [ksplit * T, E], summed by the router kernel in split order."""
    if logits.is_cuda and kind == "sigmoid":
        t = logits.shape[0] // ksplit
        ids = torch.empty(t, topk, dtype=torch.int32, device=logits.device)
        w = torch.empty(t, topk, dtype=torch.float32, device=logits.device)
        ext().moe_route(logits.float().contiguous(), e_bias.float().contiguous(), ids, w, n_group, topk_group,
                        routed_scale, ksplit)
        return ids, w
    if ksplit > 1:
        logits = logits.view(ksplit, -1, logits.shape[1]).sum(0)
    return route_ref(logits, e_bias, topk, n_group, topk_group, routed_scale, kind)


def route_fuses_splitk(num_experts: int, n_group: int, kind: str = "sigmoid") -> bool:
    """The router kernel sums split-K partials itself for this geometry (its register form)."""
    return kind == "sigmoid" and num_experts % 32 == 0 and num_experts <= 256 and (num_experts // n_group) % 32 == 0


def _topk_stable(x: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest per row; ties go to the lower index (stable descending sort)."""
    return torch.sort(x, dim=-1, descending=True, stable=True).indices[..., :k]


def route_ref(logits: torch.Tensor, e_bias: torch.Tensor, topk: int, n_group: int, topk_group: int,
              routed_scale: float, kind: str = "sigmoid") -> tuple[torch.Tensor, torch.Tensor]:
    logits = logits.float()
    t, e = logits.shape
    if kind == "softmax":
        p = torch.softmax(logits, dim=-1)
        ids = _topk_stable(p, topk)
        w = p.gather(1, ids)
        return ids.int(), w / w.sum(-1, keepdim=True)
    scores = torch.sigmoid(logits)
    sel = scores + e_bias.float()[None, :]
    if n_group > 1:
        g = sel.view(t, n_group, e // n_group)
        gscore = g.sort(dim=-1, descending=True).values[..., :2].sum(-1)
        keep = _topk_stable(gscore, topk_group)
        mask = torch.zeros(t, n_group, dtype=torch.bool, device=logits.device)
        mask.scatter_(1, keep, True)
        sel = sel.masked_fill(~mask.repeat_interleave(e // n_group, dim=1), float("-inf"))
    ids = _topk_stable(sel, topk)
    w = scores.gather(1, ids)
    w = w / w.sum(-1, keepdim=True).clamp(min=1e-20) * routed_scale
    return ids.int(), w


def swiglu(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    from .basic import act_mul
    return Fn.linear(act_mul(Fn.linear(x, w_gu), gelu=False), w_down)


def moe_forward(x: torch.Tensor, gate: torch.Tensor, e_bias: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
                shared_gu: torch.Tensor, shared_down: torch.Tensor, topk: int, n_group: int, topk_group: int,
                routed_scale: float, kind: str = "sigmoid") -> torch.Tensor:
    """x bf16 [T, H]; w_gu [E, 2F, H]; w_down [E, H, F]; shared_* one shared expert (or None).  Dropless: every
    (token, expert) pair is computed; contributions are summed in fp32 in expert order then added to the shared
    expert's output."""
    logits = Fn.linear(x.float(), gate.float())
    ids, w = route(logits, e_bias, topk, n_group, topk_group, routed_scale, kind)
    out = experts_ref(x, ids, w, w_gu, w_down, 0)
    if shared_gu is not None:
        out += swiglu(x, shared_gu, shared_down).float()
    return out.to(torch.bfloat16)


def experts_ref(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
                e0: int) -> torch.Tensor:
    """fp32 [T, H] sum over the (token, slot) pairs routed to experts e0 .. e0 + len(w_gu) - 1 (expert order) of
    weight * SwiGLU expert output; other ids (and -1) contribute nothing."""
    t, topk = ids.shape
    out = torch.zeros(t, x.shape[1], dtype=torch.float32, device=x.device)
    flat = ids.long().view(-1) - e0
    keep = (flat >= 0) & (flat < w_gu.shape[0])
    flat = torch.where(keep, flat, torch.full_like(flat, w_gu.shape[0]))
    order = torch.argsort(flat, stable=True)
    experts, counts = torch.unique_consecutive(flat[order], return_counts=True)
    start = 0
    for e, c in zip(experts.tolist(), counts.tolist()):
        sel = order[start:start + c]
        start += c
        if e >= w_gu.shape[0]:
            continue
        rows = sel // topk
        y = swiglu(x[rows], w_gu[e], w_down[e])
        out.index_add_(0, rows, y.float() * w.view(-1)[sel, None])
    return out


def piggyback_pack(scales: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, kmax: int) -> torch.Tensor:
    """Routing that rides in the activation-scale tensor of a DP gather (one collective instead of two,
    `moe-gemm/router-piggyback/dp_router_piggyback.py:1-25`): [rows, G] fp32 scales + top-k ids (as exact fp32
    integers) + weights -> [rows, G + 2 kmax]; unused slots id -1, weight 0."""
    rows, k = ids.shape
    out = torch.zeros(rows, scales.shape[1] + 2 * kmax, dtype=torch.float32, device=scales.device)
    out[:, :scales.shape[1]] = scales.float()
    g = scales.shape[1]
    out[:, g:g + kmax] = -1.0
    out[:, g:g + k] = ids.float()
    out[:, g + kmax:g + kmax + k] = w.float()
    return out


def piggyback_unpack(packed: torch.Tensor, groups: int, kmax: int, k: int):
    """Inverse of piggyback_pack -> (scales [rows, G], ids int32 [rows, k], weights [rows, k])."""
    return (packed[:, :groups], packed[:, groups:groups + k].round().int(),
            packed[:, groups + kmax:groups + kmax + k])
