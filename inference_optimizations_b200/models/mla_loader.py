"""HuggingFace checkpoints for the MLA + DSA + MoE family (DeepSeek-V3 / V3.2 layout, GLM-5 class): a weight source
for `MLAModel(source=...)` and the inverse export.

The model fetches every tensor by its own weight name (`MLAModel._make_layer`); `HFMLASource` maps that name to the
checkpoint tensor(s) it is made of (`hf_names`), reads them from the safetensors shards (one tensor at a time, so a
node-size model never sits on the host twice), dequantizes FP8 E4M3 weights stored with a per-128x128-block
`weight_scale_inv` (the DeepSeek-V3 FP8 checkpoint format), concatenates gate / up projections, and returns bf16 on
the model's device; the model then packs it for its kernels and drops it.  Expert-parallel ranks ask only for their
experts, so each rank reads only its share of the routed experts.

Rotary dims: the DeepSeek checkpoints store the q / k rope dims in interleaved pair order while this framework rotates
halves (NeoX); `rope_interleaved=True` permutes those rows (pairs (0, 1), (2, 3), ... -> halves), which leaves every
q.k product unchanged.  `index_rope_interleaved` does the same for the indexer's rope dims (the first qk_rope dims of
each index head and of the index key).

Names follow the HuggingFace DeepSeek-V3 modelling files (`model.layers.{i}.self_attn.q_a_proj.weight`, ...; the MTP
layer is `model.layers.{num_layers}` with `eh_proj`, `enorm`, `hnorm`, `shared_head.norm`) and the V3.2 indexer
(`self_attn.indexer.{wq_b, wk, k_norm, weights_proj}`); the reference serves the same checkpoints through SGLang's
loader (its DSA patches, `parallelism/dsa-decode-context-parallel/0002-*.patch`).
"""
from __future__ import annotations

import glob
import json
import os
from typing import Optional

import torch

from .loader import SafeTensors, save

_ATTN = {"wq_a": "self_attn.q_a_proj.weight", "q_norm": "self_attn.q_a_layernorm.weight",
         "wq_b": "self_attn.q_b_proj.weight", "wkv_a": "self_attn.kv_a_proj_with_mqa.weight",
         "kv_norm": "self_attn.kv_a_layernorm.weight", "wkv_b": "self_attn.kv_b_proj.weight",
         "wo": "self_attn.o_proj.weight", "wi_q": "self_attn.indexer.wq_b.weight",
         "wi_k": "self_attn.indexer.wk.weight", "wi_kn": "self_attn.indexer.k_norm.weight",
         "wi_kb": "self_attn.indexer.k_norm.bias", "wi_w": "self_attn.indexer.weights_proj.weight",
         "n_in": "input_layernorm.weight", "n_post": "post_attention_layernorm.weight",
         "gate": "mlp.gate.weight", "e_bias": "mlp.gate.e_score_correction_bias",
         "shared.down": "mlp.shared_experts.down_proj.weight", "mlp.down": "mlp.down_proj.weight"}
_PAIRS = {"shared.gu": ("mlp.shared_experts.gate_proj.weight", "mlp.shared_experts.up_proj.weight"),
          "mlp.gu": ("mlp.gate_proj.weight", "mlp.up_proj.weight")}


def hf_names(name: str, num_layers: int) -> list:
    """This model's weight name -> the checkpoint tensor name(s) it is made of (concatenated along dim 0)."""
    L = f"model.layers.{num_layers}."
    top = {"embed": ["model.embed_tokens.weight"], "lm_head": ["lm_head.weight"], "final_norm": ["model.norm.weight"],
           "mtp.eh_proj": [L + "eh_proj.weight"], "mtp.enorm": [L + "enorm.weight"], "mtp.hnorm": [L + "hnorm.weight"],
           "mtp.norm": [L + "shared_head.norm.weight"]}
    if name in top:
        return top[name]
    parts = name.split(".")
    if parts[0] == "mtp":                    # "mtp.<i>.<suffix>": the draft layer, index i = num_layers
        parts = parts[1:]
    layer, suffix = parts[0], ".".join(parts[1:])
    base = f"model.layers.{int(layer)}."
    if suffix in _ATTN:
        return [base + _ATTN[suffix]]
    if suffix in _PAIRS:
        return [base + n for n in _PAIRS[suffix]]
    if suffix.startswith("experts.gu."):
        e = suffix.rsplit(".", 1)[1]
        return [base + f"mlp.experts.{e}.gate_proj.weight", base + f"mlp.experts.{e}.up_proj.weight"]
    if suffix.startswith("experts.down."):
        return [base + f"mlp.experts.{suffix.rsplit('.', 1)[1]}.down_proj.weight"]
    raise KeyError(f"no checkpoint name for weight {name!r}")


def _halves_perm(d: int) -> torch.Tensor:
    """Row order taking interleaved rotary pairs (x0, x1), (x2, x3), ... to rotate-half layout [x0 x2 ..| x1 x3 ..]."""
    return torch.cat([torch.arange(0, d, 2), torch.arange(1, d, 2)])


def dequant_fp8_blocks(w: torch.Tensor, scale_inv: torch.Tensor, block: int = 128) -> torch.Tensor:
    """FP8 E4M3 [N, K] with one fp32 scale per 128 x 128 block ([ceil(N/128), ceil(K/128)]) -> fp32."""
    N, K = w.shape
    s = scale_inv.float().repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return w.float() * s


def quant_fp8_blocks(w: torch.Tensor, block: int = 128) -> tuple:
    """bf16 / fp32 [N, K] -> (E4M3 [N, K], fp32 scale_inv per 128 x 128 block): amax / 448 per block."""
    N, K = w.shape
    nb, kb = -(-N // block), -(-K // block)
    pad = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    pad[:N, :K] = w.float()
    blk = pad.view(nb, block, kb, block)
    amax = blk.abs().amax(dim=(1, 3)).clamp(min=1e-12)
    scale = amax / 448.0
    q = (blk / scale[:, None, :, None]).view(nb * block, kb * block)[:N, :K].to(torch.float8_e4m3fn)
    return q, scale


class HFMLASource:
    """Weight source over a directory (or list) of safetensors shards in the DeepSeek-V3 layout."""

    def __init__(self, path, cfg, device, rope_interleaved: bool = True, index_rope_interleaved: bool = False):
        files = sorted(glob.glob(os.path.join(path, "*.safetensors"))) if isinstance(path, str) else list(path)
        if not files:
            raise FileNotFoundError(f"no .safetensors under {path}")
        self.cfg, self.device = cfg, torch.device(device)
        self.rope_interleaved, self.index_rope_interleaved = rope_interleaved, index_rope_interleaved
        self.where: dict = {}
        self.files = [SafeTensors(f) for f in files]
        for st in self.files:
            for k in st.keys():
                self.where[k] = st

    def close(self) -> None:
        for st in self.files:
            st.close()

    def _read(self, hf: str) -> torch.Tensor:
        if hf not in self.where:
            raise KeyError(f"checkpoint has no tensor {hf!r}")
        t = self.where[hf].get(hf)
        if t.dtype == torch.float8_e4m3fn:
            sname = hf + "_scale_inv"
            if sname not in self.where:
                raise KeyError(f"FP8 tensor {hf!r} without its block scales {sname!r}")
            return dequant_fp8_blocks(t, self.where[sname].get(sname))
        return t.float()

    def _rope_rows(self, name: str, t: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        suffix = name.split(".")[-1]
        r = c.qk_rope
        if self.rope_interleaved and suffix == "wq_b":
            t = t.view(c.num_heads, c.qk_nope + c.qk_rope, -1)
            t = torch.cat([t[:, :c.qk_nope], t[:, c.qk_nope:][:, _halves_perm(r)]], 1).reshape(-1, t.shape[-1])
        elif self.rope_interleaved and suffix == "wkv_a":
            t = torch.cat([t[:c.kv_lora], t[c.kv_lora:][_halves_perm(r)]])
        elif self.index_rope_interleaved and suffix == "wi_q":
            t = t.view(c.index_heads, c.index_dim, -1)
            t = torch.cat([t[:, :r][:, _halves_perm(r)], t[:, r:]], 1).reshape(-1, t.shape[-1])
        elif self.index_rope_interleaved and suffix == "wi_k":
            t = torch.cat([t[:r][_halves_perm(r)], t[r:]])
        return t

    def tensor(self, name: str, shape, std: float = 0.0) -> torch.Tensor:
        t = torch.cat([self._read(n) for n in hf_names(name, self.cfg.num_layers)])
        t = self._rope_rows(name, t)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} != model shape {tuple(shape)}")
        return t.to(torch.bfloat16).to(self.device)

    def norm(self, name: str, n: int, fill: float, dtype=torch.bfloat16) -> torch.Tensor:
        names = hf_names(name, self.cfg.num_layers)
        if names[0] not in self.where and name.endswith(("e_bias", "wi_kb")):
            return torch.full((n,), fill, dtype=dtype, device=self.device)     # optional in older checkpoints
        t = self._read(names[0])
        if t.numel() != n:
            raise ValueError(f"{name}: checkpoint size {t.numel()} != {n}")
        return t.to(dtype).to(self.device)


def export_hf(model, path: str, fp8: bool = False, shard_bytes: int = 4 << 30,
              rope_interleaved: bool = True) -> list:
    """Write a model that kept its bf16 masters (`keep_master`, expert parallel world 1) in the checkpoint layout
    `HFMLASource` reads (the inverse mapping; with `fp8`, 2-D projection weights as E4M3 + 128 x 128 block
    `weight_scale_inv`).  -> the shard files written."""
    c = model.cfg
    if model.ep_world != 1 or model.dcp_world != 1 or not model.keep_master:
        raise ValueError("export needs a single-rank model that kept its bf16 masters")
    inv = lambda d: torch.argsort(_halves_perm(d))  # noqa: E731
    out: dict = {}

    def put(name: str, t: torch.Tensor, quant: bool = False):
        t = t.detach().float().cpu()
        suffix = name.split(".")[-1]
        if rope_interleaved and suffix == "wq_b":
            v = t.view(c.num_heads, c.qk_nope + c.qk_rope, -1)
            t = torch.cat([v[:, :c.qk_nope], v[:, c.qk_nope:][:, inv(c.qk_rope)]], 1).reshape(-1, v.shape[-1])
        elif rope_interleaved and suffix == "wkv_a":
            t = torch.cat([t[:c.kv_lora], t[c.kv_lora:][inv(c.qk_rope)]])
        names = hf_names(name, c.num_layers)
        chunks = torch.chunk(t, len(names)) if len(names) > 1 else [t]
        for n, part in zip(names, chunks):
            if quant and fp8 and part.dim() == 2:
                q, sc = quant_fp8_blocks(part)
                out[n], out[n + "_scale_inv"] = q, sc
            else:
                out[n] = part.to(torch.float32 if name.endswith("e_bias") else torch.bfloat16)

    put("embed", model.embed)
    put("lm_head", model.lm_head, True)
    put("final_norm", model.final_norm)
    for idx, w in enumerate(model.layers):
        i = idx
        pre = f"mtp.{i}" if (model.draft and idx == len(model.layers) - 1) else str(i)
        for k in ("n_in", "n_post", "q_norm", "kv_norm", "wi_kn", "wi_kb"):
            put(f"{pre}.{k}", getattr(w, k))
        for k in ("wq_a", "wq_b", "wkv_a", "wo", "wi_q", "wi_k", "wi_w"):
            put(f"{pre}.{k}", getattr(w, k), True)
        wkv_b = torch.cat([w.w_uk.float(), w.w_uv.float().transpose(1, 2)], 1)      # [H, nope + v, kv_lora]
        put(f"{pre}.wkv_b", wkv_b.reshape(-1, c.kv_lora), True)
        f = w.ffn
        if c.is_moe(i):
            put(f"{pre}.gate", f["gate"])
            put(f"{pre}.e_bias", f["e_bias"])
            if f.get("shared_gu") is not None:
                put(f"{pre}.shared.gu", f["shared_gu"], True)
                put(f"{pre}.shared.down", f["shared_down"], True)
            for e in range(f["w_gu"].shape[0]):
                put(f"{pre}.experts.gu.{e}", f["w_gu"][e], True)
                put(f"{pre}.experts.down.{e}", f["w_down"][e], True)
        else:
            put(f"{pre}.mlp.gu", f["w_gu"], True)
            put(f"{pre}.mlp.down", f["w_down"], True)
    if model.draft:
        put("mtp.eh_proj", model.eh_proj, True)
        put("mtp.enorm", model.enorm)
        put("mtp.hnorm", model.hnorm)
        put("mtp.norm", model.draft_norm)
    os.makedirs(path, exist_ok=True)
    files, cur, size, k = [], {}, 0, 0
    for n in sorted(out):
        t = out[n]
        cur[n] = t
        size += t.numel() * t.element_size()
        if size >= shard_bytes:
            files.append(os.path.join(path, f"model-{k:05d}.safetensors"))
            save(cur, files[-1])
            cur, size, k = {}, 0, k + 1
    if cur:
        files.append(os.path.join(path, f"model-{k:05d}.safetensors"))
        save(cur, files[-1])
    with open(os.path.join(path, "config.json"), "w") as fh:
        json.dump({"architectures": ["DeepseekV32ForCausalLM"], "num_hidden_layers": c.num_layers,
                   "hidden_size": c.hidden, "num_attention_heads": c.num_heads, "q_lora_rank": c.q_lora,
                   "kv_lora_rank": c.kv_lora, "qk_nope_head_dim": c.qk_nope, "qk_rope_head_dim": c.qk_rope,
                   "v_head_dim": c.v_head, "n_routed_experts": c.num_experts, "num_experts_per_tok": c.topk,
                   "moe_intermediate_size": c.expert_ffn, "intermediate_size": c.dense_ffn,
                   "first_k_dense_replace": c.first_dense, "vocab_size": c.vocab, "index_n_heads": c.index_heads,
                   "index_head_dim": c.index_dim, "index_topk": c.index_topk,
                   "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128]} if fp8 else None},
                  fh, indent=1)
    return files


def load_mla(path: str, cfg, device, ep_rank: int = 0, ep_world: int = 1, keep_master: Optional[bool] = None,
             rope_interleaved: bool = True, index_rope_interleaved: bool = False, draft: bool = False, **kw):
    """An `MLAModel` with the checkpoint's weights (this EP rank's experts only; with `draft`, the MTP layer too)."""
    from .mla import MLAModel
    src = HFMLASource(path, cfg, device, rope_interleaved, index_rope_interleaved)
    try:
        m = MLAModel(cfg, device, ep_rank=ep_rank, ep_world=ep_world, keep_master=keep_master, source=src, **kw)
        if draft:
            m.build_draft()
        return m
    finally:
        src.close()
