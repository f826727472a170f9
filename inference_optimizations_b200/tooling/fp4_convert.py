"""INT4 (QAT, group-32 symmetric, compressed-tensors "pack-quantized") expert weights -> NVFP4 or MXFP4, with the
per-block scale chosen by squared-error search so each FP4 block is the closest one to the INT4 reference
(`moe-gemm/int4-to-nvfp4-converter/k27_fp4_convert.py:1-30`).

Layouts written:
  nvfp4  ModelOpt: `weight` uint8 [out, in/2] (E2M1 pairs, low nibble first), `weight_scale` E4M3 [out, in/16],
         `weight_scale_2` fp32 (global), `input_scale` fp32 when supplied; dequant = e2m1 * scale * global
  mxfp4  `weight` uint8 [out, in/2], `weight_scale` uint8 E8M0 [out, in/32]; dequant = e2m1 * 2^(e - 127)
E2M1 rounding is to nearest with ties to even (the hardware conversion).  The NVFP4 candidates are amax/6 times
1 .. 7/6 in 8 steps, each rounded to what the E4M3 scale can store; MXFP4 candidates are the power of two at or
above amax/6 and its two neighbours.

    python -m inference_optimizations_b200.tooling.fp4_convert convert --src DIR --dst DIR --fmt nvfp4

Per-tensor errors against the INT4 reference (weight space and output space) go to fp4_convert_stats.json.
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Optional

import torch

from ..ops import formats as F

GROUP_INT4 = 32
_LEVELS = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def unpack_int4(packed: torch.Tensor, cols: int) -> torch.Tensor:
    """int32 [out, ceil(in/8)] (nibble i of a word = column 8k + i, stored with a +8 offset) -> int8 [out, in]."""
    parts = [((packed >> (4 * i)) & 0xF) for i in range(8)]
    u = torch.stack(parts, dim=-1).reshape(packed.shape[0], -1)[:, :cols]
    return (u - 8).to(torch.int8)


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """Inverse of unpack_int4 (for tests and synthetic checkpoints)."""
    out, cols = codes.shape
    pad = (-cols) % 8
    u = torch.nn.functional.pad(codes.int() + 8, (0, pad)).reshape(out, -1, 8)
    w = torch.zeros(out, u.shape[1], dtype=torch.int64)
    for i in range(8):
        w |= (u[..., i].long() & 0xF) << (4 * i)
    return w.to(torch.int64).where(w < 2 ** 31, w - 2 ** 32).to(torch.int32)


def dequant_int4(packed: torch.Tensor, scale: torch.Tensor, cols: int) -> torch.Tensor:
    q = unpack_int4(packed, cols).float()
    return q * scale.float().repeat_interleave(GROUP_INT4, dim=1)[:, :cols]


def _round_e2m1(y: torch.Tensor) -> torch.Tensor:
    """Signed values -> nearest E2M1 value (ties to even, saturating at 6)."""
    mag = F._e2m1_mag_even(y.abs())
    return torch.where(y < 0, -_LEVELS.to(y.device)[mag], _LEVELS.to(y.device)[mag])


def _codes(y: torch.Tensor) -> torch.Tensor:
    mag = F._e2m1_mag_even(y.abs())
    return mag | (((y < 0) & (mag > 0)).int() << 3)


def _pick(blocks: torch.Tensor, cands: torch.Tensor) -> torch.Tensor:
    """blocks [.., nb, B], candidate scales [.., nb, C] (> 0) -> the scale with the least squared error."""
    errs = []
    for c in range(cands.shape[-1]):
        s = cands[..., c:c + 1]
        errs.append(((_round_e2m1(blocks / s) * s - blocks) ** 2).sum(-1))
    best = torch.stack(errs, -1).argmin(-1, keepdim=True)
    return cands.gather(-1, best).squeeze(-1)


def quant_nvfp4(w: torch.Tensor, search: bool = True, global_scale: Optional[float] = None):
    """fp32 [out, in] -> (weight uint8 [out, in/2], weight_scale E4M3 [out, in/16], weight_scale_2 fp32 [])."""
    out, cols = w.shape
    blocks = w.float().reshape(out, cols // 16, 16)
    amax = blocks.abs().amax(-1)
    g = max(float(global_scale) if global_scale else float(w.abs().max()) / (6.0 * 448.0), 1e-12)
    steps = torch.linspace(1.0, 7.0 / 6.0, 8, device=w.device) if search else torch.ones(1, device=w.device)
    cands = (amax / 6.0)[..., None] * steps
    cands = (cands / g).clamp(max=448.0).to(torch.float8_e4m3fn).float() * g       # storable scales only
    cands = torch.where(cands > 0, cands, torch.full_like(cands, g))
    s = _pick(blocks, cands) if search else cands[..., 0]
    codes = _codes(blocks / s[..., None]).reshape(out, cols)
    return F.pack_nibbles(codes), (s / g).to(torch.float8_e4m3fn), torch.tensor(g, dtype=torch.float32)


def dequant_nvfp4(weight: torch.Tensor, weight_scale: torch.Tensor, weight_scale_2: torch.Tensor) -> torch.Tensor:
    vals = F.e2m1_decode(F.unpack_nibbles(weight))
    return vals * (weight_scale.float() * float(weight_scale_2)).repeat_interleave(16, dim=1)


def quant_mxfp4(w: torch.Tensor, search: bool = True):
    """fp32 [out, in] -> (weight uint8 [out, in/2], weight_scale E8M0 uint8 [out, in/32])."""
    out, cols = w.shape
    blocks = w.float().reshape(out, cols // 32, 32)
    amax = blocks.abs().amax(-1).clamp(min=1e-30)
    p = torch.exp2(torch.ceil(torch.log2(amax / 6.0)))
    s = _pick(blocks, torch.stack([p / 2, p, p * 2], -1)) if search else p
    codes = _codes(blocks / s[..., None]).reshape(out, cols)
    e = (torch.log2(s).round() + 127).clamp(0, 254).to(torch.uint8)
    return F.pack_nibbles(codes), e


def dequant_mxfp4(weight: torch.Tensor, weight_scale: torch.Tensor) -> torch.Tensor:
    vals = F.e2m1_decode(F.unpack_nibbles(weight))
    return vals * torch.exp2(weight_scale.float() - 127.0).repeat_interleave(32, dim=1)


def compare(ref: torch.Tensor, cand: torch.Tensor, n_act: int = 256, seed: int = 0) -> dict:
    """Relative RMS error in weight space and in output space (Gaussian activations), max abs, changed fraction."""
    d = cand - ref
    x = torch.randn(n_act, ref.shape[1], generator=torch.Generator().manual_seed(seed)).to(ref.device)
    return {"rel_rms_w": float(d.norm() / ref.norm()), "rel_rms_out": float((x @ d.T).norm() / (x @ ref.T).norm()),
            "max_abs": float(d.abs().max()), "changed_frac": float((d != 0).float().mean())}


def _int4_groups(names) -> dict:
    """{prefix: {packed, scale, shape}} for compressed-tensors pack-quantized weights."""
    out = {}
    for n in names:
        for suf, key in ((".weight_packed", "packed"), (".weight_scale", "scale"), (".weight_shape", "shape")):
            if n.endswith(suf):
                out.setdefault(n[: -len(suf)], {})[key] = n
    return {k: v for k, v in out.items() if len(v) == 3}


def convert_file(src: str, dst: str, fmt: str, search: bool = True, input_scales: Optional[dict] = None) -> dict:
    """Convert every INT4 group of one safetensors file; other tensors pass through unchanged."""
    from ..models.loader import SafeTensors, save
    st = SafeTensors(src)
    names = st.keys()
    groups = _int4_groups(names)
    used = {n for g in groups.values() for n in g.values()}
    tensors, stats = {}, {}
    for n in names:
        if n not in used:
            tensors[n] = st.get(n)
    for prefix, g in groups.items():
        shape = [int(v) for v in st.get(g["shape"]).tolist()]
        ref = dequant_int4(st.get(g["packed"]), st.get(g["scale"]), shape[1])
        if fmt == "nvfp4":
            q, s8, g2 = quant_nvfp4(ref, search)
            tensors[prefix + ".weight"] = q
            tensors[prefix + ".weight_scale"] = s8
            tensors[prefix + ".weight_scale_2"] = g2.reshape(1)
            if input_scales and prefix in input_scales:
                tensors[prefix + ".input_scale"] = input_scales[prefix].reshape(1).float()
            deq = dequant_nvfp4(q, s8, g2)
        else:
            q, e8 = quant_mxfp4(ref, search)
            tensors[prefix + ".weight"] = q
            tensors[prefix + ".weight_scale"] = e8
            deq = dequant_mxfp4(q, e8)
        stats[prefix] = compare(ref, deq)
    save(tensors, dst)
    return stats


def convert(src_dir: str, dst_dir: str, fmt: str, search: bool = True) -> dict:
    """Stream a checkpoint directory shard by shard (one shard in memory at a time)."""
    os.makedirs(dst_dir, exist_ok=True)
    stats = {}
    for f in sorted(os.listdir(src_dir)):
        if f.endswith(".safetensors"):
            stats.update(convert_file(os.path.join(src_dir, f), os.path.join(dst_dir, f), fmt, search))
    with open(os.path.join(dst_dir, "fp4_convert_stats.json"), "w") as fh:
        json.dump({"fmt": fmt, "search": search, "tensors": stats}, fh, indent=1)
    return stats


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("convert")
    c.add_argument("--src", required=True)
    c.add_argument("--dst", required=True)
    c.add_argument("--fmt", choices=["nvfp4", "mxfp4"], default="nvfp4")
    c.add_argument("--no-search", action="store_true")
    a = ap.parse_args()
    if a.cmd == "convert":
        s = convert(a.src, a.dst, a.fmt, not a.no_search)
        worst = max((v["rel_rms_w"] for v in s.values()), default=0.0)
        print(json.dumps({"tensors": len(s), "worst_rel_rms_w": worst}))


if __name__ == "__main__":
    main()
