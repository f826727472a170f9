"""Dense GQA decoder with interleaved sliding-window / global layers (Gemma class, 31B), tensor parallel.

Per layer (Gemma-3 block): x = norm_in(h); qkv = x W_qkv; q, k = qk-norm + RoPE; k, v -> paged pool (fused kernel);
a = attention(q, pool); o = a W_o (TP all-reduce); h += norm_post_attn(o); x = norm_pre_ffn(h);
f = (gelu_tanh(x W_g) * x W_u) W_d (TP all-reduce); h += norm_post_ffn(f).  Norms use the (1 + w) convention,
embeddings are scaled by sqrt(hidden) and tied to the LM head.  Sliding layers see 1024 keys (q - kv < 1024), the
rule of `attention/extend-gqa/extend_attention_gqa.py:18-24`; head_dim 256 on sliding layers, 512 on global layers.

Tensor parallel (tp ranks): q/k/v heads and FFN columns are split across ranks (column-parallel W_qkv, W_gu;
row-parallel W_o, W_d followed by an all-reduce), the vocabulary of the LM head is split and the greedy token is the
max over ranks of the local argmax.  Weights are random-init (seeded) or loaded from HF safetensors (`loader.py`).

The draft head for speculative decoding (EAGLE-style, one sliding-window layer, `speculative/` in the reference)
shares the embedding / LM head: x = W_fc [emb(token); h_prev] -> layer -> norm -> logits.

On a GPU every projection and the LM head run on this framework's weight-streaming tcgen05 GEMM (`ops/linear.py`,
bf16 packed weights); with tensor parallelism and a push-form `parallel.symm.TPComm`, W_o and W_d are the fused
GEMM -> all-reduce: the GEMM's epilogue stores each output tile into every rank's symmetric buffer and one kernel sums
the slots locally and applies the norm chain.  The bf16 masters are kept only for small models (the cache-free
oracle and checkpoint export read them).
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch
import torch.nn.functional as Fn

from ..config import GQAConfig
from ..ops import attention as A
from ..ops import basic as B
from ..ops import kvcache as K
from ..ops import linear as L


def _randn(shape, std, gen, device, dtype=torch.bfloat16):
    t = torch.empty(shape, dtype=dtype, device=device)
    # fill in slices so a 30 GB model never needs a second fp32 copy
    flat = t.view(-1)
    step = 1 << 26
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = (torch.randn(n, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)
    return t


@dataclass
class LayerWeights:
    qkv: torch.Tensor
    o: torch.Tensor
    gu: torch.Tensor
    down: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    n_in: torch.Tensor
    n_post_attn: torch.Tensor
    n_pre_ffn: torch.Tensor
    n_post_ffn: torch.Tensor


@dataclass
class LayerGeom:
    head_dim: int
    kv_heads: int        # local
    q_heads: int         # local
    window: int          # 0 = global
    kind: str            # "global" | "swa"


class GQAModel:
    def __init__(self, cfg: GQAConfig, device, tp_rank: int = 0, tp: int = 1, seed: int = 0,
                 all_reduce: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 weights: Optional[dict] = None, draft: bool = False, keep_master: Optional[bool] = None):
        """keep_master: keep the bf16 weights next to the GEMM's packed copies on a GPU (default: models under 2 G
        parameters; the cache-free oracle and checkpoint export need them)."""
        self.cfg, self.device, self.tp_rank, self.tp = cfg, torch.device(device), tp_rank, tp
        self.all_reduce = all_reduce
        self.tp_comm = None          # parallel.symm.TPComm: fused peer-memory all-reduce + norms (tp > 1)
        if cfg.num_q_heads % tp or cfg.num_kv_heads % tp or cfg.num_kv_heads_global % tp or cfg.ffn % tp:
            raise ValueError(f"tp={tp} does not divide the head / ffn counts")
        self.hidden = cfg.hidden
        self.ffn_local = cfg.ffn // tp
        self.vocab_local = cfg.vocab // tp
        n_layers = cfg.draft_layers if draft else cfg.num_layers
        self.geoms = []
        for i in range(n_layers):
            glob = (not draft) and cfg.is_global(i)
            d = cfg.head_dim_global if glob else cfg.head_dim
            hk = (cfg.num_kv_heads_global if glob else cfg.num_kv_heads) // tp
            self.geoms.append(LayerGeom(d, hk, cfg.num_q_heads // tp, 0 if glob else cfg.sliding_window,
                                        "global" if glob else ("draft" if draft else "swa")))
        std = cfg.init_std
        h = cfg.hidden
        if weights is None:
            # TP-invariant random init: every weight is generated as `nb` canonical blocks along its sharded
            # dimension, each from its own seed, and a rank generates only the blocks it owns.  Any tp dividing nb
            # therefore assembles exactly the same full model.
            nb = next(n for n in (8, 4, 2, 1) if cfg.num_q_heads % n == 0 and cfg.num_kv_heads % n == 0
                      and cfg.num_kv_heads_global % n == 0 and cfg.ffn % n == 0 and cfg.vocab % n == 0)
            if nb % tp:
                raise ValueError(f"tp={tp} does not divide the {nb} canonical weight blocks")
            own = range(tp_rank * nb // tp, (tp_rank + 1) * nb // tp)
            tag = f"{seed}/{'draft' if draft else 'main'}"

            def blocks(name, shape, blk_ids, dim):
                parts = []
                for b in blk_ids:
                    g = torch.Generator(device=self.device)
                    g.manual_seed(zlib.crc32(f"{tag}/{name}/{b}".encode()))
                    parts.append(_randn(shape, std, g, self.device))
                return parts[0] if len(parts) == 1 else torch.cat(parts, dim=dim)

            zeros = lambda n: torch.zeros(n, dtype=torch.bfloat16, device=self.device)  # noqa: E731
            self.embed = None if draft else blocks("embed", (cfg.vocab // nb, h), range(nb), 0)
            self.layers = []
            for i, g in enumerate(self.geoms):
                d, hq_b, hk_b, f_b = g.head_dim, cfg.num_q_heads // nb, g.kv_heads * tp // nb, cfg.ffn // nb
                qkv = torch.cat([blocks(f"{i}.q", (hq_b * d, h), own, 0), blocks(f"{i}.k", (hk_b * d, h), own, 0),
                                 blocks(f"{i}.v", (hk_b * d, h), own, 0)], 0)
                gu = torch.cat([blocks(f"{i}.gate", (f_b, h), own, 0), blocks(f"{i}.up", (f_b, h), own, 0)], 0)
                self.layers.append(LayerWeights(
                    qkv=qkv, o=blocks(f"{i}.o", (h, hq_b * d), own, 1), gu=gu,
                    down=blocks(f"{i}.down", (h, f_b), own, 1),
                    q_norm=zeros(d), k_norm=zeros(d),
                    n_in=zeros(h), n_post_attn=zeros(h), n_pre_ffn=zeros(h), n_post_ffn=zeros(h)))
            self.final_norm = torch.zeros(h, dtype=torch.bfloat16, device=self.device)
            self.fc = blocks("fc", (h, 2 * h), [0], 0) if draft else None
        else:
            self._adopt(weights, draft)
        self.rope = {}
        self.embed_scale = math.sqrt(h) if cfg.embed_scale else 1.0
        self.keep_master = keep_master if keep_master is not None else cfg.num_params() < 2e9
        self._build_linears()

    def _build_linears(self) -> None:
        """Pack every projection (and this rank's LM-head rows) for the weight-streaming GEMM; without keep_master
        the bf16 masters are dropped as each is packed, so a node-size model holds one copy."""
        self.lins, self.head = None, None
        if self.device.type != "cuda":
            return

        def mk(w):
            return L.Linear(w, "bf16") if w.shape[1] % 64 == 0 else None

        self.lins = []
        for w in self.layers:
            d = {}
            for name in ("qkv", "o", "gu", "down"):
                d[name] = mk(getattr(w, name))
                if d[name] is not None and not self.keep_master:
                    setattr(w, name, None)
            self.lins.append(d)
        if self.embed is not None:
            lo = self.tp_rank * self.vocab_local
            self.head = mk(self.embed[lo:lo + self.vocab_local])

    def can_push(self) -> bool:
        """Every row-parallel projection (W_o, W_d) is on the GEMM with an unpadded output: the push form of the
        fused tensor-parallel all-reduce applies."""
        return self.lins is not None and all(d[n] is not None and d[n].Np == d[n].N
                                             for d in self.lins for n in ("o", "down"))

    def _lin(self, i: int, name: str, x: torch.Tensor, push=None) -> torch.Tensor:
        lin = self.lins[i][name] if self.lins is not None else None
        if lin is None or not x.is_cuda:
            return Fn.linear(x, getattr(self.layers[i], name))
        return lin(x, push=push)

    # ------------------------------------------------------------------------------------------------ weights
    def _adopt(self, w: dict, draft: bool) -> None:
        """Take already-sharded tensors (see loader.py) keyed by HF names."""
        h = self.cfg.hidden
        self.embed = None if draft else w["model.embed_tokens.weight"]
        self.final_norm = w["model.norm.weight"]
        self.fc = w.get("fc.weight")
        self.layers = []
        for i, g in enumerate(self.geoms):
            p = f"model.layers.{i}."
            self.layers.append(LayerWeights(
                qkv=torch.cat([w[p + "self_attn.q_proj.weight"], w[p + "self_attn.k_proj.weight"],
                               w[p + "self_attn.v_proj.weight"]], 0),
                o=w[p + "self_attn.o_proj.weight"],
                gu=torch.cat([w[p + "mlp.gate_proj.weight"], w[p + "mlp.up_proj.weight"]], 0),
                down=w[p + "mlp.down_proj.weight"],
                q_norm=w[p + "self_attn.q_norm.weight"], k_norm=w[p + "self_attn.k_norm.weight"],
                n_in=w[p + "input_layernorm.weight"], n_post_attn=w[p + "post_attention_layernorm.weight"],
                n_pre_ffn=w[p + "pre_feedforward_layernorm.weight"],
                n_post_ffn=w[p + "post_feedforward_layernorm.weight"]))
        assert all(l.qkv.shape[1] == h for l in self.layers)

    def rope_table(self, d: int, theta: float, max_pos: int) -> torch.Tensor:
        key = (d, theta)
        t = self.rope.get(key)
        if t is None or t.shape[0] < max_pos:
            t = B.rope_table(max_pos, d, theta, self.device)
            self.rope[key] = t
        return t

    def num_bytes(self) -> int:
        n = sum(t.numel() * t.element_size() for l in self.layers for t in vars(l).values() if t is not None)
        if self.lins is not None:
            n += sum(lin.lin.wpack.numel() for d in self.lins for name, lin in d.items()
                     if lin is not None and getattr(self.layers[0], name) is None)
        if self.embed is not None:
            n += self.embed.numel() * 2
        return n

    # ------------------------------------------------------------------------------------------------ forward
    def _reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            return self.all_reduce(x)
        return x

    def layer_forward(self, i: int, x_norm: torch.Tensor, resid: torch.Tensor, st: "StepTensors",
                      kv: "GQAKVCache", layer_id: int, next_norm: Optional[torch.Tensor]) -> torch.Tensor:
        """x_norm = norm_in(h) [T, H]; resid = h (updated in place).  Returns the next layer's normed input."""
        cfg, w, g = self.cfg, self.layers[i], self.geoms[i]
        eps = cfg.rms_eps
        qkv = self._lin(i, "qkv", x_norm)
        theta = cfg.rope_theta_global if g.kind == "global" else cfg.rope_theta
        cs = self.rope_table(g.head_dim, theta, kv.max_pos)
        pool = kv.pools[layer_id]
        slot = st.slot[g.kind]
        q = K.gqa_prep(qkv, w.q_norm if cfg.qk_norm else None, w.k_norm if cfg.qk_norm else None, cs, st.pos, slot,
                       pool, kv.fmt, g.q_heads, g.kv_heads, g.head_dim, eps, True, kv.k_scale, kv.v_scale)
        if st.ext_segs is not None and kv.fmt != K.FMT_BF16 and g.head_dim in (256, 512) and q.is_cuda:
            attn = A.gqa_extend(q, pool, kv.tables[g.kind].dev, st.ext_blocks(g.q_heads // g.kv_heads, q.device),
                                g.kv_heads, kv.fmt, 1.0 / math.sqrt(g.head_dim), g.window, kv.k_scale, kv.v_scale,
                                status=kv.ext_status)
        else:
            attn = A.gqa_decode(q, pool, kv.tables[g.kind].dev, st.kv_len, st.n_q, g.kv_heads, kv.fmt,
                                1.0 / math.sqrt(g.head_dim), g.window, kv.k_scale, kv.v_scale,
                                splits=st.splits.get(g.kind), ws=kv.workspace(g.head_dim, g.kv_heads, st.lane),
                                req_idx=st.req_idx)
        if self.tp > 1 and self.tp_comm is not None and attn.shape[0] <= self.tp_comm.rows_cap:
            comm, t = self.tp_comm, attn.shape[0]
            if comm.push:
                # fused GEMM -> all-reduce: the GEMM pushes its tiles into every rank's slot; one kernel sums the
                # slots locally and applies post-norm, residual add and the next pre-norm
                self._lin(i, "o", attn.view(t, -1), push=comm)
                x = comm.reduce_norm2(t, resid, w.n_post_attn, w.n_pre_ffn, eps)
                self._lin(i, "down", B.act_mul(self._lin(i, "gu", x), gelu=True), push=comm)
                return comm.reduce_norm2(t, resid, w.n_post_ffn, next_norm, eps)
            # pull form: row-parallel GEMMs write their partials into the symmetric buffer; one kernel reduces over
            # NVLink and applies post-norm, residual add and the next pre-norm
            comm.out_buffer(t).copy_(self._lin(i, "o", attn.view(t, -1)))
            x = comm.reduce_norm2(t, resid, w.n_post_attn, w.n_pre_ffn, eps)
            comm.out_buffer(t).copy_(self._lin(i, "down", B.act_mul(self._lin(i, "gu", x), gelu=True)))
            return comm.reduce_norm2(t, resid, w.n_post_ffn, next_norm, eps)
        o = self._reduce(self._lin(i, "o", attn.view(attn.shape[0], -1)))
        o = B.rmsnorm(o, w.n_post_attn, eps, True)
        x = B.rmsnorm(o, w.n_pre_ffn, eps, True, residual=resid)          # resid += o; x = norm(resid)
        f = self._reduce(self._lin(i, "down", B.act_mul(self._lin(i, "gu", x), gelu=True)))
        f = B.rmsnorm(f, w.n_post_ffn, eps, True)
        return B.rmsnorm(f, next_norm, eps, True, residual=resid)       # resid += f; x = norm_next(resid)

    def forward(self, st: "StepTensors", kv: "GQAKVCache", layer_offset: int = 0,
                inputs_embeds: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Returns (final-normed hidden [T, H], pre-norm residual stream [T, H])."""
        return self.forward_layers(st, kv, 0, len(self.layers), None, None, layer_offset, inputs_embeds)

    def forward_layers(self, st: "StepTensors", kv: "GQAKVCache", lo: int, hi: int, x: Optional[torch.Tensor],
                       resid: Optional[torch.Tensor], layer_offset: int = 0,
                       inputs_embeds: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Decoder layers [lo, hi) of one step: the split prefill of the SM-partitioned prefill / decode lanes
        (`parallelism/in-node-pd-disaggregation/glm_pdmux_split_hooks.py:1-30`).  lo == 0 embeds; (x, resid) carry
        the normed input and the residual stream between ranges; after the last layer x is final-normed."""
        cfg = self.cfg
        if lo == 0:
            resid = B.embed(st.ids, self.embed, self.embed_scale) if inputs_embeds is None else inputs_embeds
            x = B.rmsnorm(resid, self.layers[0].n_in, cfg.rms_eps, True)
        for i in range(lo, hi):
            nxt = self.layers[i + 1].n_in if i + 1 < len(self.layers) else self.final_norm
            x = self.layer_forward(i, x, resid, st, kv, layer_offset + i, nxt)
        return x, resid

    def logits_local(self, x_final: torch.Tensor, embed: torch.Tensor) -> torch.Tensor:
        if self.head is not None and embed is self.embed and x_final.is_cuda:
            return self.head(x_final)
        lo = self.tp_rank * self.vocab_local
        return Fn.linear(x_final, embed[lo:lo + self.vocab_local])

    @torch.no_grad()
    def reference_logits(self, tokens: list) -> torch.Tensor:
        """Cache-free fp32-attention forward of one sequence (tp = 1): logits [T, V].  The oracle for engine tests:
        same op sequence and bf16 rounding points, dense causal attention instead of the paged kernel."""
        from ..ops.attention import dense_attention_ref
        from ..ops.kvcache import _head_rmsnorm
        cfg, eps = self.cfg, self.cfg.rms_eps
        if self.layers and self.layers[0].qkv is None:
            raise RuntimeError("reference_logits needs the bf16 masters (GQAModel(keep_master=True))")
        t = len(tokens)
        ids = torch.tensor(tokens, dtype=torch.int32, device=self.device)
        pos = torch.arange(t, device=self.device)
        resid = B.embed(ids, self.embed, self.embed_scale)
        x = B.rmsnorm(resid, self.layers[0].n_in, eps, True)
        for i, (w, g) in enumerate(zip(self.layers, self.geoms)):
            qkv = Fn.linear(x, w.qkv).float().reshape(t, -1, g.head_dim)
            theta = cfg.rope_theta_global if g.kind == "global" else cfg.rope_theta
            cs = self.rope_table(g.head_dim, theta, t + 64)
            q = B.apply_rope_ref(_head_rmsnorm(qkv[:, :g.q_heads], w.q_norm, eps, True), pos, cs)
            k = B.apply_rope_ref(_head_rmsnorm(qkv[:, g.q_heads:g.q_heads + g.kv_heads], w.k_norm, eps, True), pos, cs)
            v = qkv[:, g.q_heads + g.kv_heads:]
            q, k, v = (z.to(torch.bfloat16).float() for z in (q, k, v))
            a = dense_attention_ref(q, k, v, 1.0 / math.sqrt(g.head_dim), pos, pos, g.window)
            o = Fn.linear(a.to(torch.bfloat16).reshape(t, -1), w.o)
            o = B.rmsnorm(o, w.n_post_attn, eps, True)
            x = B.rmsnorm(o, w.n_pre_ffn, eps, True, residual=resid)
            f = Fn.linear(B.act_mul(Fn.linear(x, w.gu), gelu=True), w.down)
            f = B.rmsnorm(f, w.n_post_ffn, eps, True)
            nxt = self.layers[i + 1].n_in if i + 1 < len(self.layers) else self.final_norm
            x = B.rmsnorm(f, nxt, eps, True, residual=resid)
        return Fn.linear(x, self.embed).float()


@dataclass
class StepTensors:
    """Device inputs of one forward step (fixed addresses when captured in a CUDA graph)."""
    ids: torch.Tensor                 # int32 [T]
    pos: torch.Tensor                 # int32 [T]
    slot: dict                        # kind -> int32 [T] pool slot (-1 = no write)
    kv_len: torch.Tensor              # int32 [B] per group
    req_idx: torch.Tensor             # int32 [B] page-table row per group
    n_q: int
    splits: dict = field(default_factory=dict)   # kind -> (num_splits, tiles_per_split) or None
    # prefill: [(first q row, real tokens, position of the first token, page-table row)] per segment; attention then
    # runs the GQA-packed extend kernel over NVFP4 / FP8 pools (block lists cached per group size G)
    ext_segs: Optional[list] = None
    ext_cache: dict = field(default_factory=dict)
    lane: int = 0                     # 1 = the prefill lane of the SM-partitioned lanes (its own decode workspace)

    def ext_blocks(self, g: int, device) -> torch.Tensor:
        if g not in self.ext_cache:
            blk = A.extend_blocks(self.ext_segs, g)
            t = torch.tensor(blk, dtype=torch.int32).reshape(-1, 4)
            self.ext_cache[g] = t.pin_memory().to(device, non_blocking=True) if torch.device(device).type == "cuda" \
                else t
        return self.ext_cache[g]


class GQAKVCache:
    """Paged KV pools of all layers + page tables.  Kinds: "global" (full-context layers), "swa" (sliding-window
    layers, pages released behind the window) and "draft" (the draft head's sliding-window layer)."""

    def __init__(self, cfg: GQAConfig, tp: int, device, fmt: str, max_requests: int, max_seq: int,
                 global_pages: int, swa_pages: int, draft_pages: int = 0, k_scale: float = 1.0,
                 v_scale: float = 1.0):
        from ..kv.allocator import PageAllocator, PageTable
        self.cfg, self.fmt_name, self.fmt = cfg, fmt, K.FMT_IDS[fmt]
        self.device = torch.device(device)
        self.max_pos = max_seq + 64
        self.k_scale, self.v_scale = k_scale, v_scale
        max_pages = (max_seq + 63) // 64 + 1
        self.pools = []
        self.kinds = []
        for i in range(cfg.num_layers):
            glob = cfg.is_global(i)
            d = cfg.head_dim_global if glob else cfg.head_dim
            hk = (cfg.num_kv_heads_global if glob else cfg.num_kv_heads) // tp
            n = global_pages if glob else swa_pages
            self.pools.append(torch.zeros(n, hk, 2, K.part_bytes(self.fmt, d), dtype=torch.uint8, device=device))
            self.kinds.append("global" if glob else "swa")
        if draft_pages:
            for _ in range(cfg.draft_layers):
                self.pools.append(torch.zeros(draft_pages, cfg.num_kv_heads // tp, 2, K.part_bytes(self.fmt, cfg.head_dim),
                                              dtype=torch.uint8, device=device))
                self.kinds.append("draft")
        self.alloc = {"global": PageAllocator(global_pages), "swa": PageAllocator(swa_pages)}
        self.tables = {"global": PageTable(max_requests, max_pages, device), "swa": PageTable(max_requests, max_pages, device)}
        if draft_pages:
            self.alloc["draft"] = PageAllocator(draft_pages)
            self.tables["draft"] = PageTable(max_requests, max_pages, device)
        self._ws = {}
        self.ext_status = torch.zeros(1, dtype=torch.int32, device=device)

    def workspace(self, d: int, hk: int, lane: int = 0) -> Optional[A.DecodeWorkspace]:
        """The decode lane's reserved split workspace; the prefill lane (lane 1) gets None, so each call allocates
        its own on the prefill stream and the two lanes never share partial buffers."""
        return self._ws.get((d, hk)) if lane == 0 else None

    def reserve_workspace(self, max_groups: int, max_splits: int) -> None:
        if self.device.type != "cuda":
            return
        for i, p in enumerate(self.pools):
            hk = p.shape[1]
            d = {K.FMT_NVFP4: p.shape[3] * 16 // (64 * 9), K.FMT_FP8: p.shape[3] // 64,
                 K.FMT_BF16: p.shape[3] // 128}[self.fmt]
            key = (d, hk)
            need = max_groups * hk * max_splits * 16
            if key not in self._ws or self._ws[key].lse_part.numel() < need:
                self._ws[key] = A.DecodeWorkspace.allocate(max_groups, hk, max_splits, d, device=self.device)

    def sync_tables(self) -> None:
        for t in self.tables.values():
            t.sync()

    def bytes_per_token(self) -> float:
        tot = 0.0
        for p, kind in zip(self.pools, self.kinds):
            if kind == "global":
                tot += p[0].numel() / 64
        return tot
