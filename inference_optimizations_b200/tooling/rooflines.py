"""Per-step rooflines at served shapes: for every op the floor max(HBM bytes / bandwidth, FLOPs / tensor peak), and
the NVLink floor of the collectives, per GPU (the reference's `tooling/rooflines/*_roofline.py` method,
`pro_roofline.py:1-35`, `glm_roofline.py:1-60`).  Peaks come from MEASURED_PEAKS.json (copy bandwidth, cuBLAS bf16)
when present, else an earlier measurement on this kind of B200 (6.65 TB/s, 1.59 PFLOP/s); NVLink uses the measured 770
GB/s per direction per GPU.

    python -m inference_optimizations_b200.tooling.rooflines --model gemma31b --batch 32 --ctx 32768 --tp 1
    python -m inference_optimizations_b200.tooling.rooflines --model dsa_moe --batch 64 --ctx 8192 --ep 8
"""
from __future__ import annotations

import argparse
import json
import os
from dataclasses import dataclass

from ..config import GQAConfig, MLAMoEConfig, model_config

# without MEASURED_PEAKS.json: an earlier copy-bandwidth / cuBLAS measurement on this kind of B200 (not the nominal
# 7.7 TB/s / 2.25 PFLOP/s, which no kernel reaches)
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "nvlink_gbs": 770.0}
KV_BYTES = {"bf16": 2.0, "fp8": 1.0, "nvfp4": 0.5 + 1.0 / 16}      # per element incl. block scales


def peaks() -> dict:
    p = dict(FALLBACK)
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        p.update({k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops") if k in d})
        p["source"] = "measured"
    else:
        p["source"] = "fallback"
    return p


@dataclass
class Op:
    name: str
    bytes: float
    flops: float
    nvlink_bytes: float = 0.0
    fp8: bool = False

    def floor_us(self, pk: dict) -> float:
        tensor = pk["bf16_tflops"] * (2 if self.fp8 else 1)
        return max(self.bytes / (pk["hbm_gbs"] * 1e3), self.flops / (tensor * 1e6)) + \
            self.nvlink_bytes / (pk["nvlink_gbs"] * 1e3)


def gqa_decode_ops(cfg: GQAConfig, batch: int, ctx: int, kv: str, tp: int) -> list:
    h, ops = cfg.hidden, []
    kvb = KV_BYTES[kv]
    for i in range(cfg.num_layers):
        glob = cfg.is_global(i)
        d = cfg.head_dim_global if glob else cfg.head_dim
        hk = (cfg.num_kv_heads_global if glob else cfg.num_kv_heads) // tp
        hq = cfg.num_q_heads // tp
        w = (h * (hq + 2 * hk) * d + hq * d * h + 3 * h * cfg.ffn // tp) * 2
        span = ctx if glob else min(ctx, cfg.sliding_window)
        kv_bytes = batch * span * hk * 2 * d * kvb
        ops.append(Op(f"L{i}.gemms", w, 2 * batch * w / 2))
        ops.append(Op(f"L{i}.attn_{'global' if glob else 'swa'}", kv_bytes, 4 * batch * span * hq * d))
        if tp > 1:
            ops.append(Op(f"L{i}.allreduce", 0, 0, nvlink_bytes=2 * batch * h * 2 * (tp - 1)))
    ops.append(Op("lm_head", cfg.vocab // tp * h * 2, 2 * batch * cfg.vocab // tp * h))
    return ops


def mla_decode_ops(cfg: MLAMoEConfig, batch: int, ctx: int, kv: str, ep: int) -> list:
    """DP attention (each GPU its own `batch` sessions, attention weights replicated), experts sharded over ep."""
    h, ops = cfg.hidden, []
    row = 352 if kv == "nvfp4" else 576
    attn_w = (h * cfg.q_lora + cfg.q_lora * cfg.num_heads * (cfg.qk_nope + cfg.qk_rope) + h * (cfg.kv_lora + cfg.qk_rope)
              + cfg.kv_lora * cfg.num_heads * (cfg.qk_nope + cfg.v_head) + cfg.num_heads * cfg.v_head * h
              + cfg.q_lora * cfg.index_heads * cfg.index_dim + h * cfg.index_dim + h * cfg.index_heads)
    for i in range(cfg.num_layers):
        ops.append(Op(f"L{i}.attn_weights", attn_w, 2 * batch * attn_w, fp8=cfg.weight_dtype == "fp8"))
        ops.append(Op(f"L{i}.indexer", batch * ctx * 132, 2 * batch * ctx * cfg.index_heads * cfg.index_dim, fp8=True))
        topk = min(ctx, cfg.index_topk)
        ops.append(Op(f"L{i}.sparse_mla", batch * topk * row,
                      2 * batch * cfg.num_heads * topk * (cfg.kv_lora + cfg.qk_rope + cfg.kv_lora), fp8=True))
        if cfg.is_moe(i):
            # experts touched per GPU per step under uniform routing: of E experts, batch * ep * topk pairs leave
            # E (1 - (1 - 1/E)^pairs) distinct ones touched, 1 / ep of them local
            local = cfg.num_experts // ep
            tokens = batch * ep * cfg.topk / ep          # token-expert pairs landing on this GPU
            touched = local * (1.0 - (1.0 - 1.0 / cfg.num_experts) ** (batch * ep * cfg.topk))
            ew = max(1.0, touched) * 3 * h * cfg.expert_ffn
            sh = cfg.num_shared * 3 * h * cfg.expert_ffn
            ops.append(Op(f"L{i}.experts", ew + sh, 2 * (tokens + batch * cfg.num_shared) * 3 * h * cfg.expert_ffn,
                          nvlink_bytes=2 * batch * cfg.topk * h * (ep - 1) / ep if ep > 1 else 0.0, fp8=True))
        else:
            ops.append(Op(f"L{i}.mlp", 3 * h * cfg.dense_ffn, 2 * batch * 3 * h * cfg.dense_ffn, fp8=True))
    fp8 = cfg.weight_dtype == "fp8"
    ops.append(Op("lm_head", cfg.vocab * h * (1 if fp8 else 2), 2 * batch * cfg.vocab * h, fp8=fp8))
    return ops


def summarize(ops: list, batch: int, pk: dict) -> dict:
    floors = {o.name: o.floor_us(pk) for o in ops}
    groups: dict = {}
    for o in ops:
        key = o.name.split(".", 1)[-1]
        groups[key] = groups.get(key, 0.0) + floors[o.name]
    step = sum(floors.values())
    return {"step_floor_ms": round(step / 1e3, 3), "tok_s_ceiling_per_gpu": round(batch / (step / 1e6), 1),
            "by_op_ms": {k: round(v / 1e3, 3) for k, v in sorted(groups.items(), key=lambda kv: -kv[1])},
            "hbm_bytes_gb": round(sum(o.bytes for o in ops) / 1e9, 3), "peaks": pk}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gemma31b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--kv", default="nvfp4")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--ep", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="truncate the model to this many layers (0: all)")
    a = ap.parse_args(argv)
    cfg = model_config(a.model, **({"num_layers": a.layers} if a.layers else {}))
    ops = gqa_decode_ops(cfg, a.batch, a.ctx, a.kv, a.tp) if isinstance(cfg, GQAConfig) else \
        mla_decode_ops(cfg, a.batch, a.ctx, a.kv, a.ep)
    print(json.dumps({"model": a.model, "batch": a.batch, "ctx": a.ctx, "kv": a.kv, "tp": a.tp, "ep": a.ep,
                      **summarize(ops, a.batch, peaks())}, indent=1))


if __name__ == "__main__":
    main()
