"""MLA + DSA + MoE decoder (DeepSeek-V3.2 / GLM-5 class; BASELINE configs 3 and 5), single GPU.

Per layer (pre-norm):
  x = norm_in(h)
  attention, absorbed form: q_a = norm_q(x W_qa); q = q_a W_qb -> (q_nope [H, d_n], q_pe [H, 64] RoPE);
    kv_a = x W_kva -> latent c = norm_kv(kv_a[:512]), k_pe = RoPE(kv_a[512:]); the row (c, k_pe) goes to the latent
    pool (NVFP4 352 B or E4M3 576 B, `ops/kvcache.py mla_write`);
    DSA indexer: q_i = q_a W_iq [Hi, 128], k_i = LayerNorm(x W_ik) (RoPE on the first 64 dims of both), head weights
    x W_iw * Hi^-1/2 * 128^-1/2; k_i goes to the index pool; the top-k positions (`ops/indexer.py`) select the rows;
    q_lat[h] = q_nope[h] W_UK[h] (512 latent dims), attention over the selected rows with the 576-dim query
    (`ops/mla.py mla_decode`, V = latent), o[h] = o_lat[h] W_UV[h]; h += o W_o
  x = norm_post(h); h += FFN(x): SwiGLU for the first `first_dense` layers, routed MoE + shared expert after
  (`ops/moe.py`).
Prefill uses the same path: with sparse attention every prompt token is a query with its own top-k over its causal
prefix (its index key and latent row are written first).  Weights are random-init, seeded per tensor.
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as Fn

from ..config import MLAMoEConfig
from ..ops import basic as B
from ..ops import formats as F
from ..ops import indexer as I
from ..ops import kvcache as K
from ..ops import mla as M
from ..ops import moe as MOE


def _rand(name: str, shape, std: float, device, seed: int) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(zlib.crc32(f"{seed}/{name}".encode()))
    t = torch.empty(shape, dtype=torch.bfloat16, device=device)
    flat = t.view(-1)
    step = 1 << 26
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = (torch.randn(n, generator=g, device=device) * std).to(torch.bfloat16)
    return t


def _rand_experts(name: str, lo: int, hi: int, shape, std: float, device, seed: int) -> torch.Tensor:
    """Experts lo..hi-1 of a stacked [E, ...] expert weight, each seeded by its own name: an expert-parallel rank
    builds only its slice and every EP width builds the same model."""
    return torch.stack([_rand(f"{name}.{e}", shape, std, device, seed) for e in range(lo, hi)]) if hi > lo else \
        torch.empty(0, *shape, dtype=torch.bfloat16, device=device)


@dataclass
class MLALayerWeights:
    n_in: torch.Tensor
    n_post: torch.Tensor
    wq_a: torch.Tensor          # [q_lora, H]
    q_norm: torch.Tensor
    wq_b: torch.Tensor          # [heads * (d_n + d_r), q_lora]
    wkv_a: torch.Tensor         # [kv_lora + d_r, H]
    kv_norm: torch.Tensor
    w_uk: torch.Tensor          # [heads, d_n, kv_lora]
    w_uv: torch.Tensor          # [heads, kv_lora, d_v]
    wo: torch.Tensor            # [H, heads * d_v]
    wi_q: torch.Tensor          # [Hi * 128, q_lora]
    wi_k: torch.Tensor          # [128, H]
    wi_kn: torch.Tensor         # LayerNorm weight [128]
    wi_kb: torch.Tensor         # LayerNorm bias [128]
    wi_w: torch.Tensor          # [Hi, H]
    ffn: dict


@dataclass
class MLAStep:
    """Device inputs of one forward: T tokens of any number of requests."""
    ids: torch.Tensor           # int32 [T]
    pos: torch.Tensor           # int32 [T]
    slot: torch.Tensor          # int32 [T] latent / index pool slot of the token (-1: not written)
    limit: torch.Tensor         # int32 [T] visible positions (the token's own included)
    req_idx: torch.Tensor       # int32 [T] page-table row
    max_ctx: int                # bound on limit (fixed per CUDA graph)


class MLAKVCache:
    def __init__(self, cfg: MLAMoEConfig, device, fmt: int, rows: int, max_pages: int, pages: int,
                 extra_layers: int = 0):
        self.cfg, self.device, self.fmt = cfg, torch.device(device), fmt
        rb = M.ROW_BYTES[fmt]
        n = cfg.num_layers + extra_layers           # extra: the MTP draft layer's pools (same page ids)
        self.latent = [torch.zeros(pages * 64, rb, dtype=torch.uint8, device=self.device) for _ in range(n)]
        self.index = [torch.zeros(pages, K.INDEX_PAGE_BYTES, dtype=torch.uint8, device=self.device)
                      for _ in range(n)]
        from ..kv.allocator import PageAllocator, PageTable
        self.alloc = PageAllocator(pages)
        self.table = PageTable(rows, max_pages, self.device)
        self.mla_ws: dict = {}
        self.idx_ws: dict = {}

    def bytes_per_token(self) -> int:
        return self.cfg.num_layers * (M.ROW_BYTES[self.fmt] + F.INDEX_ROW_BYTES)


class MLAModel:
    def __init__(self, cfg: MLAMoEConfig, device, seed: int = 0, ep_rank: int = 0, ep_world: int = 1):
        """ep_world > 1: this rank holds routed experts [ep_rank E / ep_world, (ep_rank + 1) E / ep_world) of every
        MoE layer (plus the shared expert); attention, router and dense layers are replicated."""
        self.cfg, self.device = cfg, torch.device(device)
        h, c = cfg.hidden, cfg
        if c.num_experts % ep_world:
            raise ValueError("experts must divide evenly over the expert-parallel ranks")
        self.ep_rank, self.ep_world = ep_rank, ep_world
        e_lo, e_hi = ep_rank * c.num_experts // ep_world, (ep_rank + 1) * c.num_experts // ep_world
        self.ep = None                                   # set by attach_ep(): per-layer expert-parallel MoE
        std = c.init_std
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=self.device)  # noqa: E731
        r = lambda name, shape, s=std: _rand(name, shape, s, self.device, seed)  # noqa: E731
        self.embed = r("embed", (c.vocab, h))
        self.lm_head = r("lm_head", (c.vocab, h))
        self.final_norm = ones(h)
        self.layers = []
        for i in range(c.num_layers):
            wkv_b = r(f"{i}.wkv_b", (c.num_heads * (c.qk_nope + c.v_head), c.kv_lora)).view(
                c.num_heads, c.qk_nope + c.v_head, c.kv_lora)
            if c.is_moe(i):
                ffn = {"gate": r(f"{i}.gate", (c.num_experts, h)),
                       "e_bias": torch.zeros(c.num_experts, dtype=torch.float32, device=self.device),
                       "w_gu": _rand_experts(f"{i}.experts.gu", e_lo, e_hi, (2 * c.expert_ffn, h), std,
                                             self.device, seed),
                       "w_down": _rand_experts(f"{i}.experts.down", e_lo, e_hi, (h, c.expert_ffn), std,
                                               self.device, seed),
                       "shared_gu": r(f"{i}.shared.gu", (2 * c.expert_ffn * c.num_shared, h)) if c.num_shared else None,
                       "shared_down": r(f"{i}.shared.down", (h, c.expert_ffn * c.num_shared)) if c.num_shared else None}
            else:
                ffn = {"w_gu": r(f"{i}.mlp.gu", (2 * c.dense_ffn, h)), "w_down": r(f"{i}.mlp.down", (h, c.dense_ffn))}
            self.layers.append(MLALayerWeights(
                n_in=ones(h), n_post=ones(h),
                wq_a=r(f"{i}.wq_a", (c.q_lora, h)), q_norm=ones(c.q_lora),
                wq_b=r(f"{i}.wq_b", (c.num_heads * (c.qk_nope + c.qk_rope), c.q_lora)),
                wkv_a=r(f"{i}.wkv_a", (c.kv_lora + c.qk_rope, h)), kv_norm=ones(c.kv_lora),
                w_uk=wkv_b[:, :c.qk_nope, :].contiguous(),
                w_uv=wkv_b[:, c.qk_nope:, :].transpose(1, 2).contiguous(),
                wo=r(f"{i}.wo", (h, c.num_heads * c.v_head)),
                wi_q=r(f"{i}.wi_q", (c.index_heads * c.index_dim, c.q_lora)),
                wi_k=r(f"{i}.wi_k", (c.index_dim, h)), wi_kn=ones(c.index_dim),
                wi_kb=torch.zeros(c.index_dim, dtype=torch.bfloat16, device=self.device),
                wi_w=r(f"{i}.wi_w", (c.index_heads, h)), ffn=ffn))
        self.rope = {}
        self.sm_scale = 1.0 / math.sqrt(c.qk_nope + c.qk_rope)
        self.n_target = c.num_layers
        self.draft = False

    def build_draft(self, seed: int = 0) -> None:
        """Multi-token-prediction draft head (DeepSeek-V3 MTP, depth 1): h'_i = W_eh [RMSNorm_e(Emb(t_{i+1}));
        RMSNorm_h(h_i)] through one more MLA + DSA + MoE layer (its own latent / index pools, index
        `num_layers`), a final norm and the shared LM head; it predicts t_{i+2}.  Weights random-init like the
        target's."""
        c, h = self.cfg, self.cfg.hidden
        r = lambda name, shape, s=c.init_std: _rand(name, shape, s, self.device, seed)  # noqa: E731
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=self.device)  # noqa: E731
        e_lo = self.ep_rank * c.num_experts // self.ep_world
        e_hi = (self.ep_rank + 1) * c.num_experts // self.ep_world
        i = c.num_layers
        # the draft layer is built exactly like a target layer with index num_layers (MoE, since i >= first_dense)
        wkv_b = r(f"mtp.{i}.wkv_b", (c.num_heads * (c.qk_nope + c.v_head), c.kv_lora)).view(
            c.num_heads, c.qk_nope + c.v_head, c.kv_lora)
        ffn = {"gate": r(f"mtp.{i}.gate", (c.num_experts, h)),
               "e_bias": torch.zeros(c.num_experts, dtype=torch.float32, device=self.device),
               "w_gu": _rand_experts(f"mtp.{i}.experts.gu", e_lo, e_hi, (2 * c.expert_ffn, h), c.init_std,
                                     self.device, seed),
               "w_down": _rand_experts(f"mtp.{i}.experts.down", e_lo, e_hi, (h, c.expert_ffn), c.init_std,
                                       self.device, seed),
               "shared_gu": r(f"mtp.{i}.shared.gu", (2 * c.expert_ffn * c.num_shared, h)) if c.num_shared else None,
               "shared_down": r(f"mtp.{i}.shared.down", (h, c.expert_ffn * c.num_shared)) if c.num_shared else None}
        self.layers.append(MLALayerWeights(
            n_in=ones(h), n_post=ones(h),
            wq_a=r(f"mtp.{i}.wq_a", (c.q_lora, h)), q_norm=ones(c.q_lora),
            wq_b=r(f"mtp.{i}.wq_b", (c.num_heads * (c.qk_nope + c.qk_rope), c.q_lora)),
            wkv_a=r(f"mtp.{i}.wkv_a", (c.kv_lora + c.qk_rope, h)), kv_norm=ones(c.kv_lora),
            w_uk=wkv_b[:, :c.qk_nope, :].contiguous(),
            w_uv=wkv_b[:, c.qk_nope:, :].transpose(1, 2).contiguous(),
            wo=r(f"mtp.{i}.wo", (h, c.num_heads * c.v_head)),
            wi_q=r(f"mtp.{i}.wi_q", (c.index_heads * c.index_dim, c.q_lora)),
            wi_k=r(f"mtp.{i}.wi_k", (c.index_dim, h)), wi_kn=ones(c.index_dim),
            wi_kb=torch.zeros(c.index_dim, dtype=torch.bfloat16, device=self.device),
            wi_w=r(f"mtp.{i}.wi_w", (c.index_heads, h)), ffn=ffn))
        self.eh_proj = r("mtp.eh_proj", (h, 2 * h))
        self.enorm, self.hnorm, self.draft_norm = ones(h), ones(h), ones(h)
        self.draft = True

    def moe_layers(self) -> list:
        """Indices of the MoE layers in forward order (the MTP draft layer last)."""
        return [i for i in range(len(self.layers)) if self.cfg.is_moe(i)]

    def attach_ep(self, group, T_max: int) -> None:
        """Route every MoE layer through expert parallelism over `group` (a collective, same order on every rank):
        the peer-memory exchange with grouped block-scaled GEMMs (`parallel/ep.py EPMoE`, one shared symmetric
        buffer) on CUDA with FP8 / NVFP4 experts, else the collective reference (`EPMoERef`, e.g. gloo on CPU)."""
        from ..parallel import ep as EP
        from ..ops.moe_gemm import BlockScaledExperts
        c = self.cfg
        self.ep, self.ep_pieces, self.ep_T_max = {}, 1, T_max
        comm = None
        cuda = self.device.type == "cuda" and c.expert_dtype in ("fp8", "nvfp4")
        for i in self.moe_layers():
            f, F = self.layers[i].ffn, c.expert_ffn
            sh = (f["shared_gu"][:F], f["shared_gu"][F:], f["shared_down"]) if f["shared_gu"] is not None else None
            if cuda:
                ex = BlockScaledExperts(f["w_gu"][:, :F], f["w_gu"][:, F:], f["w_down"], shared=sh,
                                        fmt=c.expert_dtype)
                if comm is None:
                    comm = EP.EPComm(self.ep_rank, self.ep_world, T_max, c.topk, c.hidden, F, c.expert_dtype,
                                     c.num_experts // self.ep_world, ex.has_shared, self.device, group)
                self.ep[i] = EP.EPMoE(self.ep_rank, self.ep_world, c.num_experts, T_max, c.topk, experts=ex,
                                      comm=comm)
                f["w_gu"] = f["w_down"] = None   # the packed FP8 / NVFP4 copy is the only one kept
            else:
                shared = (f["shared_gu"], f["shared_down"]) if f["shared_gu"] is not None else None
                self.ep[i] = EP.EPMoERef(self.ep_rank, self.ep_world, c.num_experts, T_max, c.topk, f["w_gu"],
                                         f["w_down"], shared, group)

    def ep_idle(self, layers: list) -> None:
        """An idle rank's part of one step: the exchange of every listed MoE layer, `ep_pieces` times, no tokens."""
        c = self.cfg
        x = torch.zeros(0, c.hidden, dtype=torch.bfloat16, device=self.device)
        ids = torch.zeros(0, c.topk, dtype=torch.int32, device=self.device)
        w = torch.zeros(0, c.topk, dtype=torch.float32, device=self.device)
        for i in layers:
            for _ in range(self.ep_pieces):
                self.ep[i].forward(x, ids, w)

    def draft_forward(self, st: "MLAStep", kv: "MLAKVCache", h_prev: torch.Tensor) -> torch.Tensor:
        """MTP head over the step's tokens: st.ids[j] = t_{i+1} for the position i of row j, h_prev[j] = the target's
        residual stream at i.  Writes the draft layer's KV at st.slot; returns final-normed hidden [T, H]."""
        c = self.cfg
        e = B.embed(st.ids, self.embed)
        x0 = torch.cat([B.rmsnorm(e, self.enorm, c.rms_eps), B.rmsnorm(h_prev, self.hnorm, c.rms_eps)], dim=-1)
        h = Fn.linear(x0, self.eh_proj)
        i = self.n_target
        x = B.rmsnorm(h, self.layers[i].n_in, c.rms_eps)
        return self.layer_forward(i, h, x, st, kv, self.draft_norm)

    def copy_from(self, other: "MLAModel") -> None:
        """Take another instance's weights (any device): device RNG streams differ, so tests that compare devices
        copy one model's weights into the other."""
        dev = self.device
        names = ["embed", "lm_head", "final_norm"]
        if self.draft and other.draft:
            names += ["eh_proj", "enorm", "hnorm", "draft_norm"]
        for name in names:
            setattr(self, name, getattr(other, name).to(dev))
        for mine, theirs in zip(self.layers, other.layers):
            for f in vars(theirs):
                v = getattr(theirs, f)
                if isinstance(v, dict):
                    setattr(mine, f, {k: (t.to(dev) if t is not None else None) for k, t in v.items()})
                else:
                    setattr(mine, f, v.to(dev))

    def rope_table(self, max_pos: int) -> torch.Tensor:
        key = max_pos
        if key not in self.rope:
            self.rope[key] = B.rope_table(max_pos, self.cfg.qk_rope, self.cfg.rope_theta, self.device)
        return self.rope[key]

    def _rope(self, x: torch.Tensor, pos: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
        """RoPE on the last dim of x [T, n, 64] (fp32 math, bf16 result)."""
        return B.apply_rope_ref(x.float(), pos, cs).to(torch.bfloat16)

    def _block_scaled(self, i: int):
        """Grouped block-scaled experts of layer i (FP8 128x128 or NVFP4, per `expert_dtype` / `weight_dtype`), built
        from the layer's weights on first use; the dense FFN of the first layers runs as one expert with every token."""
        from ..ops.moe_gemm import BlockScaledExperts
        if not hasattr(self, "_bs"):
            self._bs = {}
        if i not in self._bs:
            c, f = self.cfg, self.layers[i].ffn
            if c.is_moe(i):
                F = c.expert_ffn
                sh = None
                if f["shared_gu"] is not None:
                    sh = (f["shared_gu"][:F], f["shared_gu"][F:], f["shared_down"])
                self._bs[i] = BlockScaledExperts(f["w_gu"][:, :F], f["w_gu"][:, F:], f["w_down"], shared=sh,
                                                 fmt=c.expert_dtype)
            else:
                F = c.dense_ffn
                self._bs[i] = BlockScaledExperts(f["w_gu"][None, :F], f["w_gu"][None, F:], f["w_down"][None],
                                                 fmt=c.weight_dtype)
        return self._bs[i]

    def _quantized_ffn(self, i: int) -> bool:
        c = self.cfg
        if self.device.type != "cuda":
            return False
        if c.is_moe(i):
            return c.expert_dtype in ("fp8", "nvfp4") and c.num_shared <= 1
        return c.weight_dtype in ("fp8", "nvfp4")

    def _ffn(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c, f = self.cfg, self.layers[i].ffn
        if self.ep is not None and c.is_moe(i):
            logits = Fn.linear(x.float(), f["gate"].float())
            ids, w = MOE.route(logits, f["e_bias"], c.topk, c.n_group, c.topk_group, c.routed_scale, c.router)
            t, per = x.shape[0], self.ep_T_max
            outs = []
            for p in range(self.ep_pieces):      # every rank runs the same number of exchanges (agreed per step)
                lo, hi = min(t, p * per), min(t, (p + 1) * per)
                outs.append(self.ep[i].forward(x[lo:hi], ids[lo:hi].to(torch.int32).contiguous(), w[lo:hi]))
            return torch.cat(outs) if len(outs) > 1 else outs[0]
        if self._quantized_ffn(i):
            ex = self._block_scaled(i)
            t = x.shape[0]
            if not c.is_moe(i):
                ids = torch.zeros(t, 1, dtype=torch.int32, device=x.device)
                return ex.forward(x, ids, torch.ones(t, 1, device=x.device))
            logits = Fn.linear(x.float(), f["gate"].float())
            ids, w = MOE.route(logits, f["e_bias"], c.topk, c.n_group, c.topk_group, c.routed_scale, c.router)
            return ex.forward(x, ids, w)
        if not c.is_moe(i):
            return MOE.swiglu(x, f["w_gu"], f["w_down"])
        return MOE.moe_forward(x, f["gate"], f["e_bias"], f["w_gu"], f["w_down"], f["shared_gu"], f["shared_down"],
                               c.topk, c.n_group, c.topk_group, c.routed_scale, c.router)

    def layer_forward(self, i: int, h: torch.Tensor, x: torch.Tensor, st: MLAStep, kv: MLAKVCache,
                      next_norm: torch.Tensor) -> torch.Tensor:
        """x = norm_in(h); h updated in place.  Returns the next norm of h."""
        c, w = self.cfg, self.layers[i]
        t = x.shape[0]
        eps = c.rms_eps
        cs = self.rope_table(max(st.max_ctx, 1) + 64)
        qa = B.rmsnorm(Fn.linear(x, w.wq_a), w.q_norm, eps)
        q = Fn.linear(qa, w.wq_b).view(t, c.num_heads, c.qk_nope + c.qk_rope)
        q_nope, q_pe = q[..., :c.qk_nope], self._rope(q[..., c.qk_nope:], st.pos, cs)
        kva = Fn.linear(x, w.wkv_a)
        lat = B.rmsnorm(kva[:, :c.kv_lora].contiguous(), w.kv_norm, eps)
        k_pe = self._rope(kva[:, None, c.kv_lora:], st.pos, cs)[:, 0]
        K.mla_write(lat, k_pe.contiguous(), st.slot, kv.latent[i])
        # DSA indexer
        iq = Fn.linear(qa, w.wi_q).view(t, c.index_heads, c.index_dim)
        iq = torch.cat([self._rope(iq[..., :c.qk_rope], st.pos, cs), iq[..., c.qk_rope:]], dim=-1)
        ik = Fn.layer_norm(Fn.linear(x, w.wi_k).float(), (c.index_dim,), w.wi_kn.float(), w.wi_kb.float(), eps)
        ik = torch.cat([self._rope(ik[:, None, :c.qk_rope], st.pos, cs)[:, 0], ik[:, c.qk_rope:].to(torch.bfloat16)],
                       dim=-1)
        K.index_key_write(ik.contiguous(), st.slot, kv.index[i])
        iw = Fn.linear(x, w.wi_w).float() * (c.index_heads ** -0.5 * c.index_dim ** -0.5)
        q8, w_eff = I.indexer_q_quant(iq, iw)
        sel = I.indexer_select(q8, w_eff, kv.index[i], kv.table.dev, st.limit, c.index_topk, st.max_ctx,
                               req_idx=st.req_idx, ws=kv.idx_ws.get((t, st.max_ctx)))
        # absorbed sparse attention over the latent pool
        q_lat = torch.einsum("thn,hnk->thk", q_nope.float(), w.w_uk.float()).to(torch.bfloat16)
        qf = torch.cat([q_lat, q_pe], dim=-1).contiguous()
        o_lat = M.mla_decode(qf, kv.latent[i], sel, self.sm_scale, kv.fmt, ws=kv.mla_ws.get((t, c.index_topk)))
        o = torch.einsum("thk,hkv->thv", o_lat.float(), w.w_uv.float()).to(torch.bfloat16).reshape(t, -1)
        x2 = B.rmsnorm(Fn.linear(o, w.wo), w.n_post, eps, residual=h)        # h += attn; x2 = norm_post(h)
        f = self._ffn(i, x2)
        return B.rmsnorm(f, next_norm, eps, residual=h)                      # h += ffn; next norm

    def forward(self, st: MLAStep, kv: MLAKVCache) -> torch.Tensor:
        """-> final-normed hidden [T, H]."""
        return self.forward_hidden(st, kv)[0]

    def forward_hidden(self, st: MLAStep, kv: MLAKVCache) -> tuple[torch.Tensor, torch.Tensor]:
        """-> (final-normed hidden [T, H], residual stream after the last target layer [T, H])."""
        h = B.embed(st.ids, self.embed)
        x = B.rmsnorm(h, self.layers[0].n_in, self.cfg.rms_eps)
        n = self.n_target
        for i in range(n):
            nxt = self.layers[i + 1].n_in if i + 1 < n else self.final_norm
            x = self.layer_forward(i, h, x, st, kv, nxt)
        return x, h

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return Fn.linear(x, self.lm_head)
