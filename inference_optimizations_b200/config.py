"""Typed configuration: model architectures, engine knobs, CLI and environment overrides, dry-run resolver.

One dataclass tree replaces the reference's mix of SGLang server flags and `NUMINOUS_*` environment variables
(reference: `recipes/README.md:5-13`, `kv-cache-4bit/glm-kv4/glm_kv4.md:92-94`, `tooling/serving-gate/preflight.py:1-24`).
Every field can be set three ways, in increasing priority: preset default, environment variable `IOB_<FIELD>` (upper
case), command-line flag `--<field>` (dashes or underscores).  `resolve(..., dry_run=True)` prints the effective config,
which is the preflight idea: a flag that silently resolves to something else is visible before anything boots.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
from dataclasses import dataclass, field, fields
from typing import Any, Optional


# ------------------------------------------------------------------------------------------------ model configs


@dataclass
class GQAConfig:
    """Dense grouped-query-attention decoder with interleaved sliding-window and global layers (Gemma class).

    Layer i is global when (i + 1) % global_every == 0, else sliding-window with `sliding_window` keys visible to
    each query (a query at position q sees keys kv with q - kv < sliding_window, i.e. q - kv <= sliding_window - 1,
    the rule of `attention/extend-gqa/extend_attention_gqa.py:18-24`)."""

    name: str = "gemma31b"
    family: str = "gqa"
    num_layers: int = 60
    hidden: int = 5376
    num_q_heads: int = 32
    num_kv_heads: int = 16
    num_kv_heads_global: int = 16
    head_dim: int = 256
    head_dim_global: int = 512
    global_every: int = 6
    sliding_window: int = 1024
    ffn: int = 21504
    vocab: int = 262144
    rope_theta: float = 10000.0
    rope_theta_global: float = 1000000.0
    rms_eps: float = 1e-6
    tie_embeddings: bool = True
    embed_scale: bool = True          # multiply embeddings by sqrt(hidden)
    qk_norm: bool = True
    init_std: float = 0.02
    # speculative decoding: a 1-layer draft head that proposes `draft_tokens` tokens per step
    draft_layers: int = 1
    draft_tokens: int = 3

    def is_global(self, layer: int) -> bool:
        return (layer + 1) % self.global_every == 0

    def layer_head_dim(self, layer: int) -> int:
        return self.head_dim_global if self.is_global(layer) else self.head_dim

    def layer_kv_heads(self, layer: int) -> int:
        return self.num_kv_heads_global if self.is_global(layer) else self.num_kv_heads

    def num_params(self) -> int:
        n = self.vocab * self.hidden
        for i in range(self.num_layers):
            d = self.layer_head_dim(i)
            kvh = self.layer_kv_heads(i)
            n += self.hidden * d * (self.num_q_heads + 2 * kvh) + self.num_q_heads * d * self.hidden
            n += 3 * self.hidden * self.ffn + 4 * self.hidden
        return n


@dataclass
class MLAMoEConfig:
    """Multi-head latent attention + DeepSeek sparse attention (DSA) indexer + routed MoE (DeepSeek-V3.2 / GLM-5 class).

    KV per token and layer is one latent row: kv_lora (512) values + qk_rope (64) values, stored either as the
    576-byte FP8 row or the 352-byte NVFP4 row (`kv-cache-4bit/glm-kv4/glm_kv4.py:1-36`).  The indexer keeps one
    128-dim FP8 key + fp32 scale per token (132 B, `tooling/rooflines/glm_roofline.py:43-50`)."""

    name: str = "dsa_moe"
    family: str = "mla"
    num_layers: int = 61
    hidden: int = 7168
    num_heads: int = 128
    q_lora: int = 1536
    kv_lora: int = 512
    qk_nope: int = 128
    qk_rope: int = 64
    v_head: int = 128
    index_heads: int = 64
    index_dim: int = 128
    index_topk: int = 2048
    first_dense: int = 3
    dense_ffn: int = 18432
    num_experts: int = 256
    topk: int = 8
    num_shared: int = 1
    expert_ffn: int = 2048
    n_group: int = 8
    topk_group: int = 4
    routed_scale: float = 2.5
    router: str = "sigmoid"          # "sigmoid" (DeepSeek noaux_tc with bias) or "softmax" (top-k renormalised)
    weight_dtype: str = "fp8"        # "fp8" (128x128 block scales) | "nvfp4" (E2M1 + E4M3/16 + fp32 global) | "bf16"
    expert_dtype: str = "fp8"
    vocab: int = 129280
    rope_theta: float = 10000.0
    rms_eps: float = 1e-6
    init_std: float = 0.02
    draft_layers: int = 1
    draft_tokens: int = 1
    # hybrid linear attention (Kimi-Linear class): with kda_every = n > 0, layer i is a Kimi-delta-attention layer
    # unless (i + 1) % n == 0 (an MLA layer); KDA heads of 128 key / 128 value dims, a short causal conv of kda_conv
    # taps, low-rank (kda_rank) forget / output gates
    kda_every: int = 0
    kda_heads: int = 0
    kda_conv: int = 4
    kda_rank: int = 128

    def is_moe(self, layer: int) -> bool:
        return layer >= self.first_dense

    def is_kda(self, layer: int) -> bool:
        return self.kda_every > 0 and layer < self.num_layers and (layer + 1) % self.kda_every != 0

    def num_params(self) -> int:
        h = self.hidden
        attn = (h * self.q_lora + self.q_lora * self.num_heads * (self.qk_nope + self.qk_rope)
                + h * (self.kv_lora + self.qk_rope) + self.kv_lora * self.num_heads * (self.qk_nope + self.v_head)
                + self.num_heads * self.v_head * h
                + self.q_lora * self.index_heads * self.index_dim + h * self.index_dim + h * self.index_heads)
        n = 2 * self.vocab * h
        for i in range(self.num_layers):
            n += attn
            if self.is_moe(i):
                n += (self.num_experts + self.num_shared) * 3 * h * self.expert_ffn + h * self.num_experts
            else:
                n += 3 * h * self.dense_ffn
        return n


PRESETS: dict[str, Any] = {
    # dense GQA hd512 model (Gemma class, 31B): the tensor-parallel serving benchmark model
    "gemma31b": lambda: GQAConfig(),
    # DSA+MoE model (DeepSeek-V3-class) with FP8 128x128 block-scaled weights: the flagship serving benchmark model
    "dsa_moe": lambda: MLAMoEConfig(),
    # long-context MLA-DSA MoE (GLM-5 class) with NVFP4 experts (context-parallel decode)
    "glm5": lambda: MLAMoEConfig(name="glm5", num_layers=78, hidden=6144, num_heads=64, q_lora=2048, qk_nope=192,
                                 qk_rope=64, v_head=256, index_heads=32, num_experts=160, topk=8, expert_ffn=2048,
                                 dense_ffn=12288, n_group=1, topk_group=1, routed_scale=2.5,
                                 weight_dtype="fp8", expert_dtype="nvfp4", vocab=154880),
    # hybrid KDA + MLA + MoE (Kimi-Linear class): three KDA layers per MLA layer
    "kimi_linear": lambda: MLAMoEConfig(name="kimi_linear", num_layers=27, hidden=2304, num_heads=32, q_lora=1536,
                                        qk_nope=128, qk_rope=64, v_head=128, index_heads=32, num_experts=256, topk=8,
                                        expert_ffn=1024, first_dense=1, dense_ffn=9216, n_group=1, topk_group=1,
                                        vocab=163840, kda_every=4, kda_heads=32, kda_rank=128),
    # small shapes for tests (same code paths, tiny dims)
    "tiny_gqa": lambda: GQAConfig(name="tiny_gqa", num_layers=6, hidden=256, num_q_heads=4, num_kv_heads=2,
                                  num_kv_heads_global=2, head_dim=128, head_dim_global=256, global_every=3,
                                  sliding_window=48, ffn=512, vocab=512),
    "tiny_kda": lambda: MLAMoEConfig(name="tiny_kda", num_layers=3, hidden=256, num_heads=4, q_lora=128, kv_lora=512,
                                     qk_nope=32, qk_rope=64, v_head=32, index_heads=4, index_dim=128, index_topk=64,
                                     first_dense=1, dense_ffn=512, num_experts=8, topk=2, num_shared=1,
                                     expert_ffn=128, n_group=2, topk_group=1, vocab=512, weight_dtype="bf16",
                                     expert_dtype="bf16", kda_every=3, kda_heads=2, kda_rank=32),
    "tiny_mla": lambda: MLAMoEConfig(name="tiny_mla", num_layers=3, hidden=256, num_heads=4, q_lora=128, kv_lora=512,
                                     qk_nope=32, qk_rope=64, v_head=32, index_heads=4, index_dim=128, index_topk=64,
                                     first_dense=1, dense_ffn=512, num_experts=8, topk=2, num_shared=1,
                                     expert_ffn=128, n_group=2, topk_group=1, vocab=512, weight_dtype="bf16",
                                     expert_dtype="bf16"),
}


def model_config(name: str, **overrides) -> Any:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    cfg = PRESETS[name]()
    for k, v in overrides.items():
        if not hasattr(cfg, k):
            raise KeyError(f"{name}: no field {k!r}")
        setattr(cfg, k, v)
    return cfg


# ------------------------------------------------------------------------------------------------ engine config


@dataclass
class EngineConfig:
    model: str = "gemma31b"
    device: str = "cuda"
    seed: int = 0
    checkpoint: str = ""                 # HuggingFace safetensors directory (empty: seeded random-init weights)
    # KV pool
    page_size: int = 64
    kv_dtype: str = "nvfp4"              # "nvfp4" | "fp8" | "bf16" (GQA pools); MLA: "nvfp4" (352 B) | "fp8" (576 B)
                                         # | "kvmix" (FP8 and NVFP4 rows in one page space, per-request placement)
                                         # | "bf16" (unquantized 1152-B rows: the accuracy reference)
    kvmix_threshold: int = 262144        # kvmix: requests whose length reaches this live in NVFP4 (promoted when
                                         # they grow past it), shorter ones in FP8
    kvmix_fp8_share: float = 0.5         # kvmix: share of the pool's latent bytes given to FP8 pages
    max_running: int = 64
    max_total_tokens: int = 0            # KV pool cap in tokens; 0 = the requests' need, bounded by free memory
    mem_fraction: float = 0.90           # share of the device memory free at boot (less a reserve) the pool may take
    # scheduling
    chunked_prefill: int = 8192
    decode_burst: int = 1                # --num-continuous-decode-steps semantics (`scheduler/decode-burst/decode_burst.py`)
    burst_queue_cap: int = 2
    max_delay_passes: int = 8
    dp_pace_steps: int = 0               # DP: passes a lone continuing chunked prefill may be parked so idle decoders
                                         # run (`dp_policy.pace_decide`); 0 = off
    dp_skew_floor: int = 0               # DP: cap a rank's prefill chunk at max(floor, other ranks' extends) while
                                         # the others mostly decode (`dp_policy.skew_chunk_cap`); 0 = off
    # speculative decoding
    spec: bool = False
    draft_tokens: int = 3
    spec_policy: str = "adaptive"        # "adaptive": speculate only while it beats plain decode; "always"
    prefix_cache: bool = True            # radix prefix reuse (MLA family; sliding-window GQA models do not reuse)
    kda_state_cache: str = ""            # hybrid KDA models: "" = no prefix reuse; "fp32" | "bf16" | "fp8" = the
                                         # prefix cache also keeps each request's recurrent state at page
                                         # boundaries, stored in that row format, and restores it on a match
    kda_state_cache_max: int = 64        # recurrent-state snapshots the prefix cache keeps (least recent dropped)
    # runtime
    cuda_graphs: bool = True
    extend_kernel: bool = True           # GQA prefill over NVFP4 / FP8 pools through the 128-row extend kernel
    pdmux: bool = False                  # GQA, tp = 1, no spec: prefill and decode as lanes on disjoint SM partitions
    pdmux_budget: int = 65536            # tokens x layers the split prefill advances per engine iteration
    graph_batch_sizes: str = "1,2,4,8,16,32,64"
    # parallelism
    tp: int = 1
    dp: int = 1
    ep: int = 1
    dcp: int = 1
    fused_comm: bool = True              # own peer-memory kernels for collectives; False = NCCL baseline
    tp_push: bool = True                 # TP: row-parallel GEMMs push their tiles to every rank (fused GEMM ->
                                         # all-reduce); False = GEMM, then a pull-form reduce over NVLink
    tp_nvls: bool = False                # TP: switch-side reduction (NVLS multimem) after the GEMM instead of push
    tp_qar: bool = False                 # TP: FP8-quantized two-shot all-reduce over peer memory (half the wire
                                         # bytes, lossy; for byte-bound links) instead of the fused bf16 forms
    # diagnostics
    trace: str = ""                      # directory for the per-rank scheduler trace (JSONL); empty = off
    bounds_check: bool = False           # host-polled index checks before kernels (the IMA locator)

    def graph_sizes(self) -> list[int]:
        return [int(x) for x in self.graph_batch_sizes.split(",") if x]


def _coerce(tp: Any, raw: str) -> Any:
    if tp in (bool, "bool"):
        return raw.lower() in ("1", "true", "yes", "on")
    if tp in (int, "int"):
        return int(raw)
    if tp in (float, "float"):
        return float(raw)
    return raw


def apply_env(cfg: Any, prefix: str = "IOB_") -> list[str]:
    """Override fields from IOB_<FIELD> environment variables. Returns the names that were set."""
    hit = []
    for f in fields(cfg):
        key = prefix + f.name.upper()
        if key in os.environ:
            setattr(cfg, f.name, _coerce(f.type, os.environ[key]))
            hit.append(f.name)
    return hit


def add_cli(parser: argparse.ArgumentParser, cfg_cls=EngineConfig) -> None:
    for f in fields(cfg_cls):
        flag = "--" + f.name.replace("_", "-")
        if f.type in (bool, "bool"):
            parser.add_argument(flag, type=lambda s: s.lower() in ("1", "true", "yes", "on"), default=None)
        else:
            parser.add_argument(flag, type=str, default=None)


def resolve(argv: Optional[list[str]] = None, dry_run: bool = False) -> EngineConfig:
    """Preset defaults < IOB_* environment < CLI. With dry_run the effective config is printed as JSON."""
    p = argparse.ArgumentParser(add_help=False)
    add_cli(p)
    p.add_argument("--dry-run", action="store_true")
    ns, _ = p.parse_known_args(argv)
    cfg = EngineConfig()
    apply_env(cfg)
    for f in fields(cfg):
        v = getattr(ns, f.name, None)
        if v is not None:
            setattr(cfg, f.name, v if isinstance(v, bool) else _coerce(f.type, v))
    if dry_run or ns.dry_run:
        print(json.dumps({"engine": dataclasses.asdict(cfg),
                          "model": dataclasses.asdict(model_config(cfg.model))}, indent=1))
    return cfg
