"""MLA + DSA + MoE decoder (DeepSeek-V3.2 / GLM-5 class), single GPU.

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

On the GPU every projection runs on this framework's tcgen05 GEMMs (`ops/linear.py`), in the checkpoint's weight
format (FP8 128 x 128 block-scaled for the DeepSeek-V3 geometry, bf16 otherwise): x -> (q_a | kv_a | k_i | w_i) is
one launch, q_a -> (q_nope | q_pe | q_i) one launch (the rows of W_qb regrouped so each head's q_nope sits at a fixed
stride), the absorption products q_nope W_UK and o_lat W_UV one head-batched launch each, W_o, the router logits
(bf16 weights, fp32 out) and the LM head one launch each.  The routed experts and the dense FFNs are the grouped
block-scaled GEMMs.  Large models never hold a bf16 copy of their weights on the device: each tensor is generated,
converted and dropped (experts one at a time), so a node-size model fits the memory its packed weights need.
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
from ..ops import linear as L
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


class RandomSource:
    """Seeded random-init weights (each tensor from its own name's seed, so every parallel layout builds the same
    model); norms at their identity values."""

    def __init__(self, seed: int, device):
        self.seed, self.device = seed, torch.device(device)

    def tensor(self, name: str, shape, std: float) -> torch.Tensor:
        return _rand(name, shape, std, self.device, self.seed)

    def norm(self, name: str, n: int, fill: float, dtype=torch.bfloat16) -> torch.Tensor:
        return torch.full((n,), fill, dtype=dtype, device=self.device)


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
    k: Optional[dict] = None    # GEMM kernels of the projections (GPU); None: torch reference path
    kda: Optional[dict] = None  # a Kimi-delta-attention layer's weights (hybrid models); the MLA fields are then None


@dataclass
class MLAStep:
    """Device inputs of one forward: T tokens of any number of requests."""
    ids: torch.Tensor           # int32 [T]
    pos: torch.Tensor           # int32 [T]
    slot: torch.Tensor          # int32 [T] latent / index pool slot of the token (-1: not written)
    limit: torch.Tensor         # int32 [T] visible positions (the token's own included)
    req_idx: torch.Tensor       # int32 [T] page-table row
    max_ctx: int                # bound on limit (fixed per CUDA graph)
    pool_sel: Optional[torch.Tensor] = None   # int32 [T] kvmix pool of the token's request (0 FP8, 1 NVFP4)
    segs: Optional[list] = None               # host (first row, tokens, request row) per segment (hybrid KDA
                                              # prefill); None: every token its own request (decode)


class MLAKVCache:
    def __init__(self, cfg: MLAMoEConfig, device, fmt: int, rows: int, max_pages: int, pages: int,
                 extra_layers: int = 0, latent_div: int = 1, storage=None, mix: Optional[tuple] = None):
        """latent_div S > 1 (decode context parallelism): this rank's latent pools hold the rows it owns, 1 / S of
        the page space (pool row v at local row v // S); the index pools stay whole (every rank scores every row).
        storage(layers, pages, row_bytes) -> (pages, latent pools [pages * 64, row_bytes], index pools [pages,
        8448]): pools placed by the caller (prefill / decode disaggregation maps them from symmetric memory); it may
        lower the page count (both sides of a pair agree on one).
        mix = (pages_fp8, pages_fp4, threshold): a kvmix page space (`kv/kvmix.py`): latent rows of pages [0, P8) in
        FP8 pools (576 B), of pages [P8, P8 + P4) in NVFP4 pools (352 B, `latent4`), index pools over every page;
        `alloc` hands each request pages of one pool."""
        self.cfg, self.device, self.fmt = cfg, torch.device(device), fmt
        n = cfg.num_layers + extra_layers           # extra: the MTP draft layer's pools (same page ids)
        self.mixed = mix is not None
        self.latent4 = None
        if self.mixed:
            assert storage is None and latent_div == 1, "kvmix pools are local and whole"
            p8, p4, thr = mix
            pages = p8 + p4
            self.fmt = fmt = M.FMT_FP8
            self.latent4 = [torch.zeros(p4 * 64, M.ROW_BYTES[M.FMT_NVFP4], dtype=torch.uint8, device=self.device)
                            for _ in range(n)]
            self.split_slot = p8 * 64
            pages_fp8 = p8
        rb = M.ROW_BYTES[fmt]
        if self.mixed:
            self.latent = [torch.zeros(pages_fp8 * 64, rb, dtype=torch.uint8, device=self.device) for _ in range(n)]
            self.index = [torch.zeros(pages, K.INDEX_PAGE_BYTES, dtype=torch.uint8, device=self.device)
                          for _ in range(n)]
        elif storage is not None:
            assert latent_div == 1, "placed pools hold whole pages"
            pages, self.latent, self.index = storage(n, pages, rb)
        else:
            lat_rows = -(-pages * 64 // latent_div)
            self.latent = [torch.zeros(lat_rows, rb, dtype=torch.uint8, device=self.device) for _ in range(n)]
            self.index = [torch.zeros(pages, K.INDEX_PAGE_BYTES, dtype=torch.uint8, device=self.device)
                          for _ in range(n)]
        self.pages = pages
        # hybrid models: per request row, the recurrent state of every Kimi-delta-attention layer (conv taps, fp32
        # delta-rule state); those layers' latent / index pools are never read (one page each)
        self.kda: dict = {}
        if cfg.kda_every:
            H, D, W = cfg.kda_heads, 128, cfg.kda_conv
            for i in range(cfg.num_layers):
                if not cfg.is_kda(i):
                    continue
                z = lambda *shape: torch.zeros(*shape, dtype=torch.float32, device=self.device)  # noqa: E731
                self.kda[i] = {"csq": z(rows, H * D, W - 1), "csk": z(rows, H * D, W - 1),
                               "csv": z(rows, H * D, W - 1), "S": z(rows, H, D, D)}
                if not self.mixed and storage is None:
                    self.latent[i] = torch.zeros(64, rb, dtype=torch.uint8, device=self.device)
                    self.index[i] = torch.zeros(1, K.INDEX_PAGE_BYTES, dtype=torch.uint8, device=self.device)
        from ..kv.allocator import PageAllocator, PageTable
        if self.mixed:
            from ..kv.kvmix import KVMixPageSpace
            self.alloc = KVMixPageSpace(mix[0], mix[1], mix[2])
        else:
            self.alloc = PageAllocator(pages)
        self.table = PageTable(rows, max_pages, self.device)
        self.mla_ws: dict = {}
        self.idx_ws: dict = {}

    def reset_state(self, row: int) -> None:
        """Zero the recurrent KDA states of request row `row` (a new request taking the row)."""
        for st in self.kda.values():
            for v in st.values():
                v[row].zero_()

    def snapshot_state(self, row: int, fmt: str) -> dict:
        """Copy of request row `row`'s recurrent states (every KDA layer): the delta-rule state as rows of 128 in
        `fmt` ("fp32" kept as is, "bf16" / "fp8" through `ops/kda.py quant_state_rows`), the short conv taps fp32."""
        from ..ops import kda as KDA
        snap = {}
        for i, st in self.kda.items():
            S = st["S"][row]
            rows = S.reshape(-1, 128).clone() if fmt == "fp32" else KDA.quant_state_rows(S.reshape(-1, 128), fmt)
            snap[i] = {"S": rows, **{k: st[k][row].clone() for k in ("csq", "csk", "csv")}}
        return snap

    def restore_state(self, row: int, snap: dict, fmt: str) -> None:
        """Load a `snapshot_state` copy into request row `row`."""
        from ..ops import kda as KDA
        for i, st in self.kda.items():
            rows = snap[i]["S"]
            S = rows if fmt == "fp32" else KDA.dequant_state_rows(rows, fmt)
            st["S"][row].copy_(S.view_as(st["S"][row]))
            for k in ("csq", "csk", "csv"):
                st[k][row].copy_(snap[i][k])

    def workspaces(self, t: int, max_ctx: int, heads: int, topk: int):
        """(indexer workspace, sparse-MLA workspace) of a step with t tokens and context bound max_ctx, shared by
        every layer of the step (layers run one after another).  Made on first use outside stream capture, so a
        captured decode graph reuses the ones its eager warm-up made (no per-layer allocation or status clear in
        the graph); their status words accumulate over layers and steps (`check`).  None inside a capture that
        found none, and for prefill-sized steps (> 256 tokens: the ops allocate per call, so chunks of varying length
        hold no memory between steps)."""
        if self.device.type != "cuda" or t > 256:
            return None, None
        from ..ops.moe_gemm import LANE
        ik, mk = (t, max_ctx, LANE[0]), (t, topk, LANE[0])
        if ik not in self.idx_ws or mk not in self.mla_ws:
            if torch.cuda.is_current_stream_capturing():
                return self.idx_ws.get(ik), self.mla_ws.get(mk)
            if ik not in self.idx_ws:
                self.idx_ws[ik] = I.IndexerWorkspace.allocate(t, max_ctx, self.device)
            if mk not in self.mla_ws:
                self.mla_ws[mk] = M.MlaWorkspace.allocate(t, heads, M.mla_split_policy(t, topk)[0], self.device)
        return self.idx_ws[ik], self.mla_ws[mk]

    def check(self) -> None:
        """Raise if a bounded wait or range check of the indexer / sparse-MLA kernels recorded a non-zero status."""
        for name, d in (("indexer", self.idx_ws), ("sparse-MLA decode", self.mla_ws)):
            for key, ws in d.items():
                v = int(ws.status.item())
                if v:
                    raise RuntimeError(f"{name} workspace {key}: status {v}")

    def bytes_per_token(self) -> int:
        return self.cfg.num_layers * (M.ROW_BYTES[self.fmt] + F.INDEX_ROW_BYTES)


class MLAModel:
    def __init__(self, cfg: MLAMoEConfig, device, seed: int = 0, ep_rank: int = 0, ep_world: int = 1,
                 keep_master: Optional[bool] = None, dcp_rank: int = 0, dcp_world: int = 1, source=None):
        """ep_world > 1: this rank holds routed experts [ep_rank E / ep_world, (ep_rank + 1) E / ep_world) of every
        MoE layer (plus the shared expert); attention, router and dense layers are replicated.
        dcp_world > 1 (decode context parallelism; every rank runs the same tokens): the latent KV is sharded by the
        owner rule, the attention output is merged per head group over peer memory, W_UV / W_o are split by head
        group, the routed experts by rank (shared expert on rank 0), the dense FFNs by FFN columns; the partial
        outputs are summed by a fused all-reduce + norm (`attach_dcp`).
        keep_master: keep the bf16 weights next to the kernels' packed copies (default: only for models under 2 G
        parameters -- test-size models, whose weights `copy_from` moves between devices).
        source: where the weights come from -- `tensor(name, shape, std)` / `norm(name, n, fill, dtype)` by this
        model's weight names (default `RandomSource`; `models/mla_loader.HFMLASource` reads a HuggingFace
        DeepSeek-V3-layout checkpoint).  Each tensor is fetched, packed for the kernels and dropped in turn."""
        self.cfg, self.device = cfg, torch.device(device)
        h, c = cfg.hidden, cfg
        if ep_world > 1 and dcp_world > 1:
            raise ValueError("expert parallelism and decode context parallelism are separate deployments")
        if c.num_experts % max(ep_world, dcp_world) or c.num_heads % dcp_world or c.dense_ffn % (128 * dcp_world):
            raise ValueError("experts / heads / dense FFN columns must divide evenly over the ranks")
        self.ep_rank, self.ep_world = ep_rank, ep_world
        # a rank index only means something with context parallelism on (with dcp_world 1 every rank holds the
        # whole model: shared expert, all heads, all FFN columns)
        self.dcp_rank, self.dcp_world = (dcp_rank if dcp_world > 1 else 0), dcp_world
        self.dcp = None                                  # attach_dcp(): merge + reduce communicators
        self.dcp_push = None                             # push-form reduce for the row-parallel W_o (CUDA)
        pr, pw = (dcp_rank, dcp_world) if dcp_world > 1 else (ep_rank, ep_world)
        self.e_lo, self.e_hi = pr * c.num_experts // pw, (pr + 1) * c.num_experts // pw
        self.ep = None                                   # set by attach_ep(): per-layer expert-parallel MoE
        self.seed = seed
        self.keep_master = keep_master if keep_master is not None else c.num_params() < 2e9
        self.cuda = self.device.type == "cuda"
        self.fuse_glue = True                            # the fused attention-block glue kernels where they apply
        self.exact_attention = False                     # fp32 attention over exactly decoded rows (accuracy arm)
        self.kda_mid = None                              # speculative verify of a hybrid model: (layer, row) ->
                                                         # recurrent state after the segment's first token
        self._x8 = None                                  # (data_ptr of x, E4M3 x, scales) written by the last norm
        self._bs: dict = {}
        self.src = source if source is not None else RandomSource(seed, self.device)
        r = lambda name, shape, s=c.init_std: self.src.tensor(name, shape, s)  # noqa: E731
        self.embed = r("embed", (c.vocab, h))
        self.final_norm = self.src.norm("final_norm", h, 1.0)
        self.lm_head = r("lm_head", (c.vocab, h))
        self.head = None
        if self._kernels():
            self.head = L.Linear(self.lm_head, self._lin_kind())
            if not self.keep_master:
                self.lm_head = None
        self.layers = []
        for i in range(c.num_layers):
            self.layers.append(self._make_layer(str(i), i))
        self.rope = {}
        self.sm_scale = 1.0 / math.sqrt(c.qk_nope + c.qk_rope)
        self.n_target = c.num_layers
        self.draft = False

    # ------------------------------------------------------------------------------------------ weights
    def _lin_kind(self) -> str:
        return "fp8" if self.cfg.weight_dtype == "fp8" else "bf16"

    def _kernels(self) -> bool:
        """Projections on this framework's GEMMs: CUDA, and a weight format those GEMMs take (FP8 or bf16; the NVFP4
        weight format applies to experts only)."""
        return self.cuda and self.cfg.weight_dtype in ("fp8", "bf16")

    def _make_kda(self, prefix: str) -> dict:
        """A Kimi-delta-attention layer (hybrid models): fused q | k | v projection, output projection, the small
        projections (beta, low-rank forget gate, low-rank output gate; fused into one GEMM + one batched GEMM,
        `ops/kda.py KDASmallProjections`), causal conv taps, decay bias / log-rate, output norm."""
        from ..ops import kda as KDA
        c, h = self.cfg, self.cfg.hidden
        H, D, W, R = c.kda_heads, 128, c.kda_conv, c.kda_rank
        r = lambda name, shape, s=c.init_std: self.src.tensor(f"{prefix}.{name}", shape, s)  # noqa: E731
        f32 = lambda name, shape, s: r(name, shape, s).float()  # noqa: E731
        kd = {"w_qkv": r("kda.qkv", (3 * H * D, h)), "wo": r("kda.o", (h, H * D)),
              "small": KDA.KDASmallProjections(r("kda.b", (H, h)), r("kda.f_a", (R, h)), r("kda.f_b", (H * D, R)),
                                               r("kda.g_a", (R, h)), r("kda.g_b", (H * D, R))),
              "cwq": f32("kda.conv_q", (H * D, W), 0.5), "cwk": f32("kda.conv_k", (H * D, W), 0.5),
              "cwv": f32("kda.conv_v", (H * D, W), 0.5), "dt_bias": f32("kda.dt_bias", (H * D,), 0.1),
              "A_log": f32("kda.a_log", (H,), 0.5), "norm_w": self.src.norm(f"{prefix}.kda.norm", D, 1.0,
                                                                             torch.float32)}
        kd["small"].fuse()
        if self._kernels():
            kd["qkv"] = L.Linear(kd["w_qkv"], "bf16")
            kd["o"] = L.Linear(kd["wo"], "bf16")
            if not self.keep_master:
                kd["w_qkv"] = kd["wo"] = None
        return kd

    def _make_layer(self, prefix: str, i: int) -> "MLALayerWeights":
        """Layer i's weights (named `prefix`.*; the MTP draft layer uses prefix "mtp.<i>"), with the GEMM kernels
        built and, unless keep_master, the bf16 masters dropped."""
        c, h = self.cfg, self.cfg.hidden
        r = lambda name, shape, s=c.init_std: self.src.tensor(name, shape, s)  # noqa: E731
        nrm = lambda name, n, fill=1.0: self.src.norm(f"{prefix}.{name}", n, fill)  # noqa: E731
        if c.is_kda(i):
            return self._make_kda_layer(prefix, i, r, nrm)
        wkv_b = r(f"{prefix}.wkv_b", (c.num_heads * (c.qk_nope + c.v_head), c.kv_lora)).view(
            c.num_heads, c.qk_nope + c.v_head, c.kv_lora)
        moe = c.is_moe(i)
        F = c.expert_ffn
        shared = c.num_shared and self.dcp_rank == 0     # context parallelism: the shared expert runs on rank 0
        if moe:
            ffn = {"gate": r(f"{prefix}.gate", (c.num_experts, h)),
                   "e_bias": self.src.norm(f"{prefix}.e_bias", c.num_experts, 0.0, torch.float32),
                   "w_gu": None, "w_down": None,
                   "shared_gu": r(f"{prefix}.shared.gu", (2 * F * c.num_shared, h)) if shared else None,
                   "shared_down": r(f"{prefix}.shared.down", (h, F * c.num_shared)) if shared else None}
            if self.keep_master or not self._quantized_ffn(i):
                ffn["w_gu"] = self._experts(f"{prefix}.experts.gu", (2 * F, h))
                ffn["w_down"] = self._experts(f"{prefix}.experts.down", (h, F))
        else:
            ffn = {"w_gu": r(f"{prefix}.mlp.gu", (2 * c.dense_ffn, h)), "w_down": r(f"{prefix}.mlp.down", (h, c.dense_ffn))}
            if self.dcp_world > 1:                      # this rank's FFN columns (gate and up rows, down columns)
                D, S, rk = c.dense_ffn, self.dcp_world, self.dcp_rank
                lo, hi = rk * D // S, (rk + 1) * D // S
                ffn["w_gu"] = torch.cat([ffn["w_gu"][lo:hi], ffn["w_gu"][D + lo:D + hi]]).contiguous()
                ffn["w_down"] = ffn["w_down"][:, lo:hi].contiguous()
        w = MLALayerWeights(
            n_in=nrm("n_in", h), n_post=nrm("n_post", h),
            wq_a=r(f"{prefix}.wq_a", (c.q_lora, h)), q_norm=nrm("q_norm", c.q_lora),
            wq_b=r(f"{prefix}.wq_b", (c.num_heads * (c.qk_nope + c.qk_rope), c.q_lora)),
            wkv_a=r(f"{prefix}.wkv_a", (c.kv_lora + c.qk_rope, h)), kv_norm=nrm("kv_norm", c.kv_lora),
            w_uk=wkv_b[:, :c.qk_nope, :].contiguous(),
            w_uv=wkv_b[:, c.qk_nope:, :].transpose(1, 2).contiguous(),
            wo=r(f"{prefix}.wo", (h, c.num_heads * c.v_head)),
            wi_q=r(f"{prefix}.wi_q", (c.index_heads * c.index_dim, c.q_lora)),
            wi_k=r(f"{prefix}.wi_k", (c.index_dim, h)), wi_kn=nrm("wi_kn", c.index_dim),
            wi_kb=nrm("wi_kb", c.index_dim, 0.0),
            wi_w=r(f"{prefix}.wi_w", (c.index_heads, h)), ffn=ffn)
        del wkv_b
        if self.dcp_world > 1:                          # this rank's head group feeds a row-parallel W_UV / W_o
            Hg = c.num_heads // self.dcp_world
            g0 = self.dcp_rank * Hg
            w.w_uv = w.w_uv[g0:g0 + Hg].contiguous()
            w.wo = w.wo[:, g0 * c.v_head:(g0 + Hg) * c.v_head].contiguous()
        idx = len(self.layers)
        if self._quantized_ffn(i) and self.cuda:
            self._bs[idx] = self._build_ffn(prefix, i, ffn)
        if self._kernels():
            self._build_kernels(w)
            if not self.keep_master:
                for name in ("wq_a", "wq_b", "wkv_a", "wo", "wi_q", "wi_k", "wi_w"):
                    setattr(w, name, None)
                if self._quantized_ffn(i):
                    for k in ("w_gu", "w_down", "shared_gu", "shared_down"):
                        ffn[k] = None
        return w

    def _make_kda_layer(self, prefix: str, i: int, r, nrm) -> "MLALayerWeights":
        c, h = self.cfg, self.cfg.hidden
        if self.dcp_world > 1:
            raise NotImplementedError("hybrid KDA layers run without context parallelism")
        moe = c.is_moe(i)
        F = c.expert_ffn
        if moe:
            ffn = {"gate": r(f"{prefix}.gate", (c.num_experts, h)),
                   "e_bias": self.src.norm(f"{prefix}.e_bias", c.num_experts, 0.0, torch.float32),
                   "w_gu": None, "w_down": None,
                   "shared_gu": r(f"{prefix}.shared.gu", (2 * F * c.num_shared, h)) if c.num_shared else None,
                   "shared_down": r(f"{prefix}.shared.down", (h, F * c.num_shared)) if c.num_shared else None}
            if self.keep_master or not self._quantized_ffn(i):
                ffn["w_gu"] = self._experts(f"{prefix}.experts.gu", (2 * F, h))
                ffn["w_down"] = self._experts(f"{prefix}.experts.down", (h, F))
        else:
            ffn = {"w_gu": r(f"{prefix}.mlp.gu", (2 * c.dense_ffn, h)), "w_down": r(f"{prefix}.mlp.down", (h, c.dense_ffn))}
        none = {k: None for k in ("wq_a", "q_norm", "wq_b", "wkv_a", "kv_norm", "w_uk", "w_uv", "wo", "wi_q", "wi_k",
                                  "wi_kn", "wi_kb", "wi_w")}
        w = MLALayerWeights(n_in=nrm("n_in", h), n_post=nrm("n_post", h), ffn=ffn, kda=self._make_kda(prefix),
                            **none)
        idx = len(self.layers)
        if self._quantized_ffn(i) and self.cuda:
            self._bs[idx] = self._build_ffn(prefix, i, ffn)
            if not self.keep_master:
                for k in ("w_gu", "w_down", "shared_gu", "shared_down"):
                    ffn[k] = None
        if self._kernels() and moe and ffn.get("gate") is not None:
            w.k = {"gate": L.Linear(ffn["gate"], "bf16")}
        return w

    def _kda_attention(self, i: int, x: torch.Tensor, st: "MLAStep", kv: "MLAKVCache") -> torch.Tensor:
        """Kimi delta attention of layer i -> its output projection [T, hidden].  Recurrent states live per request
        row (`kv.kda[i]`): a step of single tokens (decode; CUDA graphs) gathers its rows' states, runs the fused
        decode kernel and scatters them back; a prefill step runs each segment's chunked prefill on that request's
        state in place (the state carries across chunks)."""
        from ..ops import kda as KDA
        c, kd = self.cfg, self.layers[i].kda
        t = x.shape[0]
        H, D = c.kda_heads, 128
        qkv = kd["qkv"](x) if "qkv" in kd else Fn.linear(x, kd["w_qkv"])
        q, k, v = (qkv[:, j * H * D:(j + 1) * H * D].contiguous() for j in range(3))
        b, f, g2 = (u.contiguous() for u in kd["small"].forward(x))
        beta = torch.sigmoid(b.float())
        S = kv.kda[i]
        args = (kd["dt_bias"], kd["A_log"])
        if st.segs is None or all(n == 1 for _r0, n, _slot in st.segs):
            rix = st.req_idx.long()
            cq, ck, cv, sv = (S[name].index_select(0, rix) for name in ("csq", "csk", "csv", "S"))
            o = KDA.kda_decode(q.reshape(t, H, D), k.reshape(t, H, D), v.reshape(t, H, D), f.reshape(t, H, D),
                               *args, beta, g2.reshape(t, H, D), kd["norm_w"], kd["cwq"], kd["cwk"], kd["cwv"],
                               cq, ck, cv, sv)
            for name, val in (("csq", cq), ("csk", ck), ("csv", cv), ("S", sv)):
                S[name].index_copy_(0, rix, val)
        else:
            o = torch.empty(t, H, D, dtype=torch.bfloat16, device=x.device)
            for r0, n, slot in st.segs:
                rows = slice(slot, slot + 1)
                # speculative verify (`kda_mid` set): the segment's first token runs alone and the state after it is
                # kept, so a rejected draft's row can be set back to it (the commit fold)
                parts = [(r0, 1), (r0 + 1, n - 1)] if self.kda_mid is not None and n > 1 else [(r0, n)]
                for a, m in parts:
                    sl = slice(a, a + m)
                    o[sl] = KDA.kda_prefill(q[sl].reshape(1, m, H, D), k[sl].reshape(1, m, H, D),
                                            v[sl].reshape(1, m, H, D), f[sl].reshape(1, m, H, D), *args,
                                            beta[sl][None], g2[sl].reshape(1, m, H, D), kd["norm_w"], kd["cwq"],
                                            kd["cwk"], kd["cwv"], S["csq"][rows], S["csk"][rows], S["csv"][rows],
                                            S["S"][rows])[0]
                    if self.kda_mid is not None and a == r0 and len(parts) > 1:
                        self.kda_mid[(i, slot)] = {name: S[name][slot].clone() for name in ("csq", "csk", "csv", "S")}
        o = o.reshape(t, H * D)
        return kd["o"](o) if "o" in kd else Fn.linear(o, kd["wo"])

    def _experts(self, name: str, shape) -> torch.Tensor:
        """This rank's routed experts [e_lo, e_hi) of a stacked expert weight (each expert fetched by its own name)."""
        if self.e_hi <= self.e_lo:
            return torch.empty(0, *shape, dtype=torch.bfloat16, device=self.device)
        return torch.stack([self.src.tensor(f"{name}.{e}", shape, self.cfg.init_std)
                            for e in range(self.e_lo, self.e_hi)])

    def _build_ffn(self, prefix: str, i: int, ffn: dict):
        """Grouped block-scaled FFN of layer i: MoE (this rank's routed experts + the shared one) or the dense FFN as
        one expert holding every token.  Experts are generated and packed one at a time unless masters are kept."""
        from ..ops.moe_gemm import BlockScaledExperts
        c = self.cfg
        if not c.is_moe(i):
            F = ffn["w_gu"].shape[0] // 2                # the FFN columns this rank holds
            return BlockScaledExperts(ffn["w_gu"][None, :F], ffn["w_gu"][None, F:], ffn["w_down"][None],
                                      fmt=c.weight_dtype)
        F = c.expert_ffn
        sh = None
        if ffn["shared_gu"] is not None:
            sh = (ffn["shared_gu"][:F], ffn["shared_gu"][F:], ffn["shared_down"])
        if ffn["w_gu"] is not None:
            return BlockScaledExperts(ffn["w_gu"][:, :F], ffn["w_gu"][:, F:], ffn["w_down"], shared=sh,
                                      fmt=c.expert_dtype)

        def gen(e):
            gu = self.src.tensor(f"{prefix}.experts.gu.{e}", (2 * F, c.hidden), c.init_std)
            d = self.src.tensor(f"{prefix}.experts.down.{e}", (c.hidden, F), c.init_std)
            return gu[:F], gu[F:], d
        return BlockScaledExperts.build(self.e_lo, self.e_hi, F, c.hidden, gen, shared=sh, fmt=c.expert_dtype,
                                        device=self.device)

    def _build_kernels(self, w: "MLALayerWeights") -> None:
        c = self.cfg
        kind = self._lin_kind()
        H, dn, dr = c.num_heads, c.qk_nope, c.qk_rope
        # W_qb rows regrouped [every head's q_nope | every head's q_pe | indexer q]: q_nope of head h of token t sits
        # at row t * stride + h of the output viewed as [*, d_n] (the head-batched W_UK product reads it in place)
        wqb = w.wq_b.view(H, dn + dr, c.q_lora)
        b_parts = [wqb[:, :dn].reshape(H * dn, c.q_lora), wqb[:, dn:].reshape(H * dr, c.q_lora), w.wi_q]
        width = sum(t.shape[0] for t in b_parts)
        unit = dn * 256 // math.gcd(dn, 256)
        pad = (-width) % unit
        if pad:
            b_parts.append(torch.zeros(pad, c.q_lora, dtype=torch.bfloat16, device=self.device))
        k = {"a": L.Linear.fuse([w.wq_a, w.wkv_a, w.wi_k, w.wi_w], kind),
             "b": L.Linear.fuse(b_parts, kind), "o": L.Linear(w.wo, kind)}
        k["b_stride"] = k["b"].Np // dn
        if dn % 64 == 0 and c.kv_lora % 128 == 0:
            k["uk"] = L.HeadBatchedLinear(w.w_uk.transpose(1, 2))           # [H, kv_lora, d_n]
        if c.v_head % 128 == 0 and c.kv_lora % 64 == 0:
            k["uv"] = L.HeadBatchedLinear(w.w_uv.transpose(1, 2))           # [H, d_v, kv_lora]
        if w.ffn.get("gate") is not None:
            k["gate"] = L.Linear(w.ffn["gate"], "bf16")
        w.k = k

    def build_draft(self, seed: int = 0) -> None:
        """Multi-token-prediction draft head (DeepSeek-V3 MTP, depth 1): h'_i = W_eh [RMSNorm_e(Emb(t_{i+1}));
        RMSNorm_h(h_i)] through one more MLA + DSA + MoE layer (its own latent / index pools, index
        `num_layers`), a final norm and the shared LM head; it predicts t_{i+2}.  Weights random-init like the
        target's."""
        c, h = self.cfg, self.cfg.hidden
        i = c.num_layers
        # the draft layer is built exactly like a target layer with index num_layers (MoE, since i >= first_dense)
        self.layers.append(self._make_layer(f"mtp.{i}", i))
        self.eh_proj = self.src.tensor("mtp.eh_proj", (h, 2 * h), c.init_std)
        self.eh = L.Linear(self.eh_proj, self._lin_kind()) if self._kernels() else None
        self.enorm, self.hnorm = self.src.norm("mtp.enorm", h, 1.0), self.src.norm("mtp.hnorm", h, 1.0)
        self.draft_norm = self.src.norm("mtp.norm", h, 1.0)
        self.draft = True

    def moe_layers(self) -> list:
        """Indices of the MoE layers in forward order (the MTP draft layer last)."""
        return [i for i in range(len(self.layers)) if self.cfg.is_moe(i)]

    def attach_ep(self, group, T_max: int) -> None:
        """Route every MoE layer through expert parallelism over `group` (a collective, same order on every rank):
        the peer-memory exchange with grouped block-scaled GEMMs (`parallel/ep.py EPMoE`, one shared symmetric
        buffer) on CUDA with FP8 / NVFP4 experts, else the collective reference (`EPMoERef`, e.g. gloo on CPU)."""
        from ..parallel import ep as EP
        c = self.cfg
        self.ep, self.ep_pieces, self.ep_T_max = {}, 1, T_max
        comm = None
        cuda = self.cuda and c.expert_dtype in ("fp8", "nvfp4")
        for i in self.moe_layers():
            f = self.layers[i].ffn
            if cuda:
                ex = self._block_scaled(i)
                if comm is None:
                    comm = EP.EPComm(self.ep_rank, self.ep_world, T_max, c.topk, c.hidden, c.expert_ffn,
                                     c.expert_dtype, c.num_experts // self.ep_world, ex.has_shared, self.device, group)
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
        h = self.eh(x0).contiguous() if self.eh is not None else Fn.linear(x0, self.eh_proj)
        i = self.n_target
        x = B.rmsnorm(h, self.layers[i].n_in, c.rms_eps)
        return self.layer_forward(i, h, x, st, kv, self.draft_norm)

    def copy_from(self, other: "MLAModel") -> None:
        """Take another instance's weights (any device; both must keep their bf16 masters): device RNG streams
        differ, so tests that compare devices copy one model's weights into the other.  Kernels are rebuilt."""
        if not (self.keep_master and other.keep_master):
            raise ValueError("copy_from needs both models to keep their bf16 master weights")
        dev = self.device
        names = ["embed", "lm_head", "final_norm"]
        if self.draft and other.draft:
            names += ["eh_proj", "enorm", "hnorm", "draft_norm"]
        for name in names:
            setattr(self, name, getattr(other, name).to(dev))
        for mine, theirs in zip(self.layers, other.layers):
            for f in vars(theirs):
                v = getattr(theirs, f)
                if f == "k" or v is None:
                    continue
                if f == "kda":
                    raise NotImplementedError("copy_from: hybrid KDA layers")
                if isinstance(v, dict):
                    setattr(mine, f, {k: (t.to(dev) if t is not None else None) for k, t in v.items()})
                else:
                    setattr(mine, f, v.to(dev))
        self._bs = {}
        if self._kernels():
            self.head = L.Linear(self.lm_head, self._lin_kind())
            if self.draft:
                self.eh = L.Linear(self.eh_proj, self._lin_kind())
            for w in self.layers:
                self._build_kernels(w)
        for i in range(len(self.layers)):
            if self.cuda and self._quantized_ffn(i):
                self._bs[i] = self._build_ffn("", i, self.layers[i].ffn)

    def rope_table(self, max_pos: int) -> torch.Tensor:
        key = max_pos
        if key not in self.rope:
            self.rope[key] = B.rope_table(max_pos, self.cfg.qk_rope, self.cfg.rope_theta, self.device)
        return self.rope[key]

    def _rope(self, x: torch.Tensor, pos: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
        """RoPE on the last dim of x [T, n, 64] (fp32 math, bf16 result)."""
        return B.apply_rope_ref(x.float(), pos, cs).to(torch.bfloat16)

    def _block_scaled(self, i: int):
        """Grouped block-scaled experts of layer i (FP8 128x128 or NVFP4, per `expert_dtype` / `weight_dtype`); the
        dense FFN of the first layers runs as one expert with every token."""
        if i not in self._bs:
            self._bs[i] = self._build_ffn("", i, self.layers[i].ffn)
        return self._bs[i]

    def _quantized_ffn(self, i: int) -> bool:
        c = self.cfg
        if self.device.type != "cuda":
            return False
        if c.is_moe(i):
            return c.expert_dtype in ("fp8", "nvfp4") and c.num_shared <= 1
        return c.weight_dtype in ("fp8", "nvfp4")

    def _router_logits(self, i: int, x: torch.Tensor) -> torch.Tensor:
        k = self.layers[i].k
        if k is not None and "gate" in k:
            return k["gate"](x, out_f32=True)
        return Fn.linear(x.float(), self.layers[i].ffn["gate"].float())

    def _route(self, i: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Router of MoE layer i -> (expert ids, weights).  On the kernels the router GEMM's split-K partials go
        straight to the router kernel, which sums them (one launch fewer than GEMM + reduction + router)."""
        c, f, k = self.cfg, self.layers[i].ffn, self.layers[i].k
        if (k is not None and "gate" in k and x.is_cuda and k["gate"].Np == k["gate"].N
                and MOE.route_fuses_splitk(c.num_experts, c.n_group, c.router)):
            part, ks = k["gate"].partials(x)
            return MOE.route(part, f["e_bias"], c.topk, c.n_group, c.topk_group, c.routed_scale, c.router, ksplit=ks)
        logits = self._router_logits(i, x)
        return MOE.route(logits, f["e_bias"], c.topk, c.n_group, c.topk_group, c.routed_scale, c.router)

    def _ffn(self, i: int, x: torch.Tensor, xq8: Optional[tuple] = None) -> torch.Tensor:
        """xq8: x block-quantized by the norm that produced it (FP8 FFN weights), or None."""
        c, f = self.cfg, self.layers[i].ffn
        if self.ep is not None and c.is_moe(i):
            ids, w = self._route(i, x)
            t, per = x.shape[0], self.ep_T_max
            outs = []
            for p in range(self.ep_pieces):      # every rank runs the same number of exchanges (agreed per step)
                lo, hi = min(t, p * per), min(t, (p + 1) * per)
                q = (xq8[0][lo:hi], xq8[1][lo:hi]) if xq8 is not None else None
                outs.append(self.ep[i].forward(x[lo:hi], ids[lo:hi].to(torch.int32).contiguous(), w[lo:hi], q))
            return torch.cat(outs) if len(outs) > 1 else outs[0]
        if self._quantized_ffn(i):
            ex = self._block_scaled(i)
            t = x.shape[0]
            if not c.is_moe(i):
                ids = torch.zeros(t, 1, dtype=torch.int32, device=x.device)
                return ex.forward(x, ids, torch.ones(t, 1, device=x.device), xq8=xq8)
            ids, w = self._route(i, x)
            return ex.forward(x, ids, w, xq8=xq8)
        if not c.is_moe(i):
            return MOE.swiglu(x, f["w_gu"], f["w_down"])
        return MOE.moe_forward(x, f["gate"], f["e_bias"], f["w_gu"], f["w_down"], f["shared_gu"], f["shared_down"],
                               c.topk, c.n_group, c.topk_group, c.routed_scale, c.router)

    def _attn_inputs(self, w: MLALayerWeights, x: torch.Tensor, t: int):
        """-> (q_a pre-norm, kv_a, k_i pre-norm, w_i, qb(q_a normed) callable): the projections of x."""
        c = self.cfg
        if w.k is not None:
            qa_, kva, ik_, iw_ = w.k["a"].split(w.k["a"](x))
        else:
            qa_, kva, ik_, iw_ = (Fn.linear(x, w.wq_a), Fn.linear(x, w.wkv_a), Fn.linear(x, w.wi_k),
                                  Fn.linear(x, w.wi_w))
        return qa_, kva, ik_, iw_

    def _q_proj(self, w: MLALayerWeights, qa: torch.Tensor, t: int):
        """q_a (normed) -> (q_lat [T, H, kv_lora] = q_nope W_UK, q_pe [T, H, d_r] pre-RoPE, q_i [T, Hi, 128])."""
        c = self.cfg
        H, dn, dr = c.num_heads, c.qk_nope, c.qk_rope
        if w.k is not None:
            yb = w.k["b"].lin(qa)                                      # full padded width: the head rows are in place
            q_nope = yb[:, :H * dn].view(t, H, dn)
            q_pe = yb[:, H * dn:H * (dn + dr)].view(t, H, dr)
            iq = yb[:, H * (dn + dr):H * (dn + dr) + c.index_heads * c.index_dim].view(t, c.index_heads, c.index_dim)
            if "uk" in w.k:
                q_lat = w.k["uk"](yb, t, row_stride=w.k["b_stride"])
            else:
                wuk = w.w_uk if w.w_uk.is_cuda else w.w_uk.to(qa.device)
                q_lat = torch.einsum("thn,hnk->thk", q_nope.float(), wuk.float()).to(torch.bfloat16)
            return q_lat, q_pe, iq
        q = Fn.linear(qa, w.wq_b).view(t, H, dn + dr)
        q_lat = torch.einsum("thn,hnk->thk", q[..., :dn].float(), w.w_uk.float()).to(torch.bfloat16)
        iq = Fn.linear(qa, w.wi_q).view(t, c.index_heads, c.index_dim)
        return q_lat, q[..., dn:], iq

    def _o_proj(self, w: MLALayerWeights, o_lat: torch.Tensor, t: int, push=None) -> torch.Tensor:
        """push: a push-form TPComm -- W_o's GEMM stores its rows into every rank's slot (fused GEMM -> all-reduce)."""
        c = self.cfg
        if w.k is not None and "uv" in w.k:
            o = w.k["uv"](o_lat, t).view(t, -1)
        else:
            wuv = w.w_uv if w.w_uv.device == o_lat.device else w.w_uv.to(o_lat.device)
            o = torch.einsum("thk,hkv->thv", o_lat.float(), wuv.float()).to(torch.bfloat16).reshape(t, -1)
        if push is not None:
            return w.k["o"](o, push=push)
        return w.k["o"](o) if w.k is not None else Fn.linear(o, w.wo)

    # ------------------------------------------------------------------------------------------ context parallel
    def attach_dcp(self, group, T_max: int) -> None:
        """Decode context parallelism over `group` (a collective; every rank runs the same tokens): on CUDA the
        owned-row decode + peer-memory merge (`parallel/dcp.DCPAttention`) and the fused peer-memory all-reduce +
        residual + norm (`parallel/symm.TPComm`); elsewhere their collective references (gloo on CPU)."""
        from ..parallel import dcp as D
        c = self.cfg
        if self.cuda:
            from ..parallel.symm import TPComm
            self.dcp = D.DCPAttention(self.dcp_rank, self.dcp_world, T_max, c.num_heads, self.device, group)
            self.dcp_comm = TPComm(self.dcp_rank, self.dcp_world, T_max, c.hidden, self.device, group)
            if all(l.k is not None and "o" in l.k and l.k["o"].Np == l.k["o"].N for l in self.layers):
                # W_o's GEMM pushes its rows to every rank (the FFN share, a combine output, uses the pull form)
                self.dcp_push = TPComm(self.dcp_rank, self.dcp_world, T_max, c.hidden, self.device, group, push=True)
        else:
            self.dcp = D.DCPAttentionRef(self.dcp_rank, self.dcp_world, c.num_heads, group)
            self.dcp_comm = None
        self.dcp_group = group

    def _dcp_reduce(self, partial: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """h += sum over ranks of partial (every rank's share of a row-parallel product); -> rmsnorm(h, norm_w)."""
        t, eps = partial.shape[0], self.cfg.rms_eps
        if self.dcp_comm is not None:
            buf = self.dcp_comm.out_buffer(t)
            if buf.data_ptr() != partial.data_ptr():
                buf.copy_(partial)
            return self.dcp_comm.reduce_norm2(t, h, None, norm_w, eps, plus_one=False)
        import torch.distributed as dist
        p32 = partial.float()
        dist.all_reduce(p32, group=self.dcp_group)
        return B.rmsnorm(p32.to(torch.bfloat16), norm_w, eps, residual=h)

    def _ffn_dcp(self, i: int, x: torch.Tensor) -> torch.Tensor:
        """This rank's share of layer i's FFN for every token: its routed experts (pairs routed elsewhere weigh 0)
        plus the shared expert on rank 0, or its dense FFN columns.  -> partial [T, H] (summed over the ranks)."""
        c, f = self.cfg, self.layers[i].ffn
        t = x.shape[0]
        if not c.is_moe(i):
            if self._quantized_ffn(i):
                ids = torch.zeros(t, 1, dtype=torch.int32, device=x.device)
                return self._block_scaled(i).forward(x, ids, torch.ones(t, 1, device=x.device))
            return MOE.swiglu(x, f["w_gu"], f["w_down"])
        ids, w = self._route(i, x)
        local = (ids >= self.e_lo) & (ids < self.e_hi)
        w = torch.where(local, w, torch.zeros_like(w))
        if self._quantized_ffn(i):
            return self._block_scaled(i).forward(x, ids.to(torch.int32).contiguous(), w, e0=self.e_lo)
        out = MOE.experts_ref(x, ids, w, f["w_gu"], f["w_down"], self.e_lo)
        if f["shared_gu"] is not None:
            out += MOE.swiglu(x, f["shared_gu"], f["shared_down"]).float()
        return out.to(torch.bfloat16)

    def _layer_forward_dcp(self, i: int, h: torch.Tensor, x: torch.Tensor, st: MLAStep, kv: MLAKVCache,
                           next_norm: torch.Tensor) -> torch.Tensor:
        """One layer under decode context parallelism: the replicated query and top-k, the latent row written by its
        owner only (pool row v -> rank v % S, local row v // S), sparse attention over the owned rows merged for
        this rank's head group, row-parallel W_UV / W_o and FFN shares summed by the fused all-reduce + norm."""
        c, w = self.cfg, self.layers[i]
        t = x.shape[0]
        S, rk = self.dcp_world, self.dcp_rank
        lat_slot = torch.where((st.slot >= 0) & (st.slot % S == rk), st.slot // S,
                               torch.full_like(st.slot, -1)).to(torch.int32)
        qf, sel = (self._query_fused if self._fused_glue(w) else self._query_torch)(i, x, st, kv, lat_slot)
        o_g = self.dcp.decode(qf, kv.latent[i], sel, self.sm_scale, kv.fmt)          # [T, H / S, 512] merged
        if self.dcp_push is not None:                                                # fused W_o -> all-reduce
            self._o_proj(w, o_g.contiguous(), t, push=self.dcp_push)
            x2 = self.dcp_push.reduce_norm2(t, h, None, w.n_post, c.rms_eps, plus_one=False)
        else:
            x2 = self._dcp_reduce(self._o_proj(w, o_g.contiguous(), t), h, w.n_post)   # h += attn; x2 = norm(h)
        return self._dcp_reduce(self._ffn_dcp(i, x2), h, next_norm)                 # h += ffn; next norm

    def _fused_glue(self, w: MLALayerWeights) -> bool:
        """The two fused glue kernels (csrc/mla_prep.cu) serve this layer: CUDA kernels for every projection, the
        head-batched W_UK product, and the DeepSeek dims those kernels are written for (rope 64, latent 512, index
        key 128)."""
        c = self.cfg
        return (self.fuse_glue and w.k is not None and "uk" in w.k and c.qk_rope == 64 and c.kv_lora == 512
                and c.index_dim == 128)

    def _query_fused(self, i: int, x: torch.Tensor, st: MLAStep, kv: MLAKVCache,
                     lat_slot: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
        """The attention block up to the sparse-attention inputs with the glue in two kernels: x -> (q_a | kv_a | k_i
        | w_i) -> [q_a norm, latent norm + k_pe RoPE + pool write, index key LayerNorm + RoPE + pool write, head
        weights]; q_a -> (q_nope | q_pe | q_i); q_nope W_UK written straight into the attention query's first 512
        columns; then [q_pe RoPE into its last 64 columns, index query RoPE + E4M3 quantization]; the indexer's
        top-k.  -> (query bf16 [T, H, 576], selected pool slots int32 [T, topk]).  lat_slot: latent pool rows when
        they differ from the token slots (context parallelism)."""
        from .._ext import ext
        c, w = self.cfg, self.layers[i]
        t, dev, eps = x.shape[0], x.device, c.rms_eps
        cs = self.rope_table(max(st.max_ctx, 1) + 64)
        x8, self._x8 = self._x8, None
        if x8 is not None and x8[0] == x.data_ptr():    # the previous norm already wrote x block-quantized
            ya = w.k["a"].lin.forward_quantized(x8[1], x8[2])
        else:
            ya = w.k["a"].lin(x)
        qa = torch.empty(t, c.q_lora, dtype=torch.bfloat16, device=dev)
        iw = torch.empty(t, c.index_heads, dtype=torch.float32, device=dev)
        fp8_b = w.k["b"].kind == "fp8" and c.q_lora % 128 == 0     # q_a leaves the kernel already block-quantized
        qa_q = torch.empty(t, c.q_lora, dtype=torch.uint8, device=dev) if fp8_b else None
        qa_s = torch.empty(t, c.q_lora // 128, dtype=torch.int32, device=dev) if fp8_b else None
        ext().mla_prep_kv(ya, w.q_norm, w.kv_norm, w.wi_kn, w.wi_kb, cs, st.pos, st.slot, qa, kv.latent[i],
                          kv.index[i], iw, c.index_heads ** -0.5 * c.index_dim ** -0.5, c.q_lora, c.index_heads, eps,
                          lat_slot, qa_q, qa_s, kv.latent4[i] if kv.mixed else None,
                          kv.split_slot if kv.mixed else 0)
        yb = w.k["b"].lin.forward_quantized(qa_q, qa_s) if fp8_b else w.k["b"].lin(qa)
        qf = torch.empty(t, c.num_heads, 576, dtype=torch.bfloat16, device=dev)
        w.k["uk"](yb, t, row_stride=w.k["b_stride"], out=qf.view(t * c.num_heads, 576)[:, :512])
        q8 = torch.empty(t, c.index_heads, c.index_dim, dtype=torch.uint8, device=dev)
        w_eff = torch.empty(t, c.index_heads, dtype=torch.float32, device=dev)
        ext().mla_prep_q(yb, cs, st.pos, qf, q8, w_eff, iw, c.num_heads, c.qk_nope, c.index_heads)
        sel = I.indexer_select(q8, w_eff, kv.index[i], kv.table.dev, st.limit, c.index_topk, st.max_ctx,
                               req_idx=st.req_idx, ws=kv.workspaces(t, st.max_ctx, c.num_heads, c.index_topk)[0])
        return qf, sel

    def _query_torch(self, i: int, x: torch.Tensor, st: MLAStep, kv: MLAKVCache,
                     lat_slot: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
        """The same as `_query_fused` through torch ops and the separate writer kernels (CPU, and shapes the fused
        kernels do not take)."""
        c, w = self.cfg, self.layers[i]
        t = x.shape[0]
        eps = c.rms_eps
        cs = self.rope_table(max(st.max_ctx, 1) + 64)
        qa_, kva, ik_, iw_ = self._attn_inputs(w, x, t)
        qa = B.rmsnorm(qa_.contiguous(), w.q_norm, eps)
        q_lat, q_pe, iq = self._q_proj(w, qa, t)
        q_pe = self._rope(q_pe, st.pos, cs)
        lat = B.rmsnorm(kva[:, :c.kv_lora].contiguous(), w.kv_norm, eps)
        k_pe = self._rope(kva[:, None, c.kv_lora:], st.pos, cs)[:, 0]
        slot = st.slot if lat_slot is None else lat_slot
        if kv.mixed:                                # kvmix: slots past the split live in the NVFP4 pool
            lo = torch.where(slot < kv.split_slot, slot, torch.full_like(slot, -1))
            hi = torch.where(slot >= kv.split_slot, slot - kv.split_slot, torch.full_like(slot, -1))
            K.mla_write(lat, k_pe.contiguous(), lo, kv.latent[i])
            K.mla_write(lat, k_pe.contiguous(), hi, kv.latent4[i])
        else:
            K.mla_write(lat, k_pe.contiguous(), slot, kv.latent[i])
        # DSA indexer
        iq = torch.cat([self._rope(iq[..., :c.qk_rope], st.pos, cs), iq[..., c.qk_rope:]], dim=-1)
        ik = Fn.layer_norm(ik_.float(), (c.index_dim,), w.wi_kn.float(), w.wi_kb.float(), eps)
        ik = torch.cat([self._rope(ik[:, None, :c.qk_rope], st.pos, cs)[:, 0], ik[:, c.qk_rope:].to(torch.bfloat16)],
                       dim=-1)
        K.index_key_write(ik.contiguous(), st.slot, kv.index[i])
        iw = iw_.float() * (c.index_heads ** -0.5 * c.index_dim ** -0.5)
        q8, w_eff = I.indexer_q_quant(iq, iw)
        sel = I.indexer_select(q8, w_eff, kv.index[i], kv.table.dev, st.limit, c.index_topk, st.max_ctx,
                               req_idx=st.req_idx, ws=kv.workspaces(t, st.max_ctx, c.num_heads, c.index_topk)[0])
        return torch.cat([q_lat, q_pe], dim=-1).contiguous(), sel

    def layer_forward(self, i: int, h: torch.Tensor, x: torch.Tensor, st: MLAStep, kv: MLAKVCache,
                      next_norm: torch.Tensor) -> torch.Tensor:
        """x = norm_in(h); h updated in place.  Returns the next norm of h."""
        if self.dcp is not None:
            return self._layer_forward_dcp(i, h, x, st, kv, next_norm)
        c, w = self.cfg, self.layers[i]
        t, eps = x.shape[0], c.rms_eps
        if w.kda is not None:                          # hybrid model: a Kimi-delta-attention layer
            return self._post_attention(i, self._kda_attention(i, x, st, kv), h, next_norm)
        qf, sel = (self._query_fused if self._fused_glue(w) else self._query_torch)(i, x, st, kv)
        # absorbed sparse attention over the latent pool
        if kv.mixed:                                # one launch per pool format over the kvmix id space
            o_lat = M.mla_decode_mixed(qf, [kv.latent[i], kv.latent4[i]], [M.FMT_FP8, M.FMT_NVFP4],
                                       [0, kv.split_slot], sel, st.pool_sel, self.sm_scale,
                                       ws=kv.workspaces(t, st.max_ctx, c.num_heads, c.index_topk)[1])
        else:
            o_lat = M.mla_decode(qf, kv.latent[i], sel, self.sm_scale, kv.fmt,
                                 ws=kv.workspaces(t, st.max_ctx, c.num_heads, c.index_topk)[1],
                                 exact=self.exact_attention)
        return self._post_attention(i, self._o_proj(w, o_lat, t), h, next_norm)

    def _post_attention(self, i: int, o: torch.Tensor, h: torch.Tensor, next_norm: torch.Tensor) -> torch.Tensor:
        """h += attention output; x2 = norm_post(h), also block-quantized when the FFN's expert GEMMs take FP8 input;
        h += FFN(x2); -> the next norm of h."""
        c, w = self.cfg, self.layers[i]
        t, eps = o.shape[0], c.rms_eps
        xq8 = None
        fp8_ffn = (self._quantized_ffn(i) and c.hidden % 128 == 0 and
                   (c.expert_dtype if c.is_moe(i) else c.weight_dtype) == "fp8")
        if fp8_ffn:
            xq8 = (torch.empty(t, c.hidden, dtype=torch.uint8, device=o.device),
                   torch.empty(t, c.hidden // 128, dtype=torch.int32, device=o.device))
        x2 = B.rmsnorm(o, w.n_post, eps, residual=h, fp8=xq8)
        f = self._ffn(i, x2, xq8)
        return self._norm_out(f, next_norm, h, i + 1)                         # h += ffn; next norm

    def _norm_out(self, f: torch.Tensor, norm_w: torch.Tensor, h: Optional[torch.Tensor], nxt: int) -> torch.Tensor:
        """rmsnorm(h + f) with h updated (or rmsnorm(f) without h); when layer `nxt` takes its input through the
        fused path with an FP8 first projection, the same kernel also writes the block-quantized copy that
        projection reads (`_x8`, consumed once by `_query_fused`)."""
        c = self.cfg
        eps = c.rms_eps
        if (nxt < self.n_target and self.cuda and c.hidden % 128 == 0 and self._fused_glue(self.layers[nxt])
                and self.layers[nxt].k["a"].kind == "fp8"):
            t = f.shape[0]
            q8 = torch.empty(t, c.hidden, dtype=torch.uint8, device=f.device)
            qs = torch.empty(t, c.hidden // 128, dtype=torch.int32, device=f.device)
            out = B.rmsnorm(f, norm_w, eps, residual=h, fp8=(q8, qs))
            self._x8 = (out.data_ptr(), q8, qs)
            return out
        return B.rmsnorm(f, norm_w, eps, residual=h)

    def forward(self, st: MLAStep, kv: MLAKVCache) -> torch.Tensor:
        """-> final-normed hidden [T, H]."""
        return self.forward_hidden(st, kv)[0]

    def forward_layers(self, st: MLAStep, kv: MLAKVCache, lo: int, hi: int, x: Optional[torch.Tensor],
                       h: Optional[torch.Tensor], x8=None) -> tuple:
        """Target layers [lo, hi) of a forward split by layer ranges (the split prefill of the SM-partitioned lanes).
        x: the normed input of layer lo (None at lo = 0: embedding and first norm here); h: the residual stream.
        x8: the block-quantized copy of x the previous range's last norm wrote for layer lo's FP8 projection.
        -> (x, h, x8) after layer hi - 1 (x is the final-normed hidden after the last layer)."""
        n = self.n_target
        if lo == 0:
            h = B.embed(st.ids, self.embed)
            x = self._norm_out(h, self.layers[0].n_in, None, 0)
        else:
            self._x8 = x8
        for i in range(lo, hi):
            nxt = self.layers[i + 1].n_in if i + 1 < n else self.final_norm
            x = self.layer_forward(i, h, x, st, kv, nxt)
        x8, self._x8 = self._x8, None
        return x, h, x8

    def forward_hidden(self, st: MLAStep, kv: MLAKVCache) -> tuple[torch.Tensor, torch.Tensor]:
        """-> (final-normed hidden [T, H], residual stream after the last target layer [T, H])."""
        h = B.embed(st.ids, self.embed)
        x = self._norm_out(h, self.layers[0].n_in, None, 0)
        n = self.n_target
        for i in range(n):
            nxt = self.layers[i + 1].n_in if i + 1 < n else self.final_norm
            x = self.layer_forward(i, h, x, st, kv, nxt)
        return x, h

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        if self.head is not None:
            return self.head(x)
        return Fn.linear(x, self.lm_head)
