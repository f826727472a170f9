"""Checkpoint converter: INT4 QAT expert weights (compressed-tensors "pack-quantized", symmetric, one scale per 32
inputs) -> NVFP4 (ModelOpt layout) or MXFP4, the weight formats this framework's block-scaled GEMMs serve
(the reference ships the same conversion for its W4A4 MoE path, `moe-gemm/int4-to-nvfp4-converter/`).

Format contracts kept as the loaders expect them:
  INT4 in   `weight_packed` int32 [out, in/8] (nibble i of a word = input column 8k + i, stored +8), `weight_scale`
            [out, in/32], `weight_shape` [2]
  nvfp4     `weight` uint8 [out, in/2] (E2M1 pairs, element 2i in the low nibble), `weight_scale` E4M3 [out, in/16],
            `weight_scale_2` fp32 (per tensor: amax / (6 * 448)), `input_scale` fp32 when supplied;
            value = e2m1 * weight_scale * weight_scale_2
  mxfp4     `weight` uint8 [out, in/2], `weight_scale` uint8 E8M0 [out, in/32]; value = e2m1 * 2^(e - 127)

Scale choice.  A block's nominal scale is amax / 6 (its largest value lands on E2M1's 6).  A storable scale is one the
format can hold: an E4M3 code times the tensor's global scale (NVFP4) or a power of two (MXFP4).  The converter takes
EVERY storable scale inside a window around the nominal one -- [amax / 8, amax / 4]: below amax / 6 the largest values
clip to 6 sigma, above it the grid coarsens -- and keeps the one whose block reconstruction has the least squared
error (ties: the smaller scale).  For NVFP4 the window spans about eight E4M3 codes (three mantissa bits per octave),
enumerated as a contiguous range of code bytes since positive E4M3 codes are ordered like their values.  Powers of two
are sparser, so MXFP4 searches [amax / 12, amax / 3]: the smallest power of two that does not clip and the one below.
All candidates of a row chunk are evaluated in one broadcast.  With `search=False` the nominal scale rounded to the
nearest storable value is used.  E2M1 rounding is to nearest, ties to even, as the
hardware conversion does.

Report (`conversion_report.json`): per tensor the signal-to-quantization-noise ratio in weight space and in output
space (against a fixed +-1 probe batch), the largest absolute error and the fraction of weights reproduced exactly.

    python -m inference_optimizations_b200.tooling.fp4_convert convert --src DIR --dst DIR --fmt nvfp4
"""
from __future__ import annotations

import argparse
import json
import math
import os
from typing import Optional

import torch

from ..ops import formats as F

GROUP_INT4 = 32
E2M1_MAX = 6.0
E4M3_MAX = 448.0
WINDOW = (1.0 / 8.0, 1.0 / 4.0)         # NVFP4 candidate scales: [amax * lo, amax * hi]
WINDOW_MX = (1.0 / 12.0, 1.0 / 3.0)     # MXFP4: a factor-of-four window (two powers of two)
_LEVELS = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
ROW_CHUNK = 256                          # rows evaluated per broadcast (bounds the candidate temporaries)


# ------------------------------------------------------------------------------------------------ INT4 input format
def unpack_int4(packed: torch.Tensor, cols: int) -> torch.Tensor:
    """int32 [out, ceil(in/8)] -> int8 [out, in] (nibble i of word k is column 8k + i, stored with a +8 offset)."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=packed.device)
    nib = (packed[..., None] >> shifts) & 0xF
    return (nib.reshape(packed.shape[0], -1)[:, :cols] - 8).to(torch.int8)


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """int8 [out, in] in [-8, 7] -> int32 [out, ceil(in/8)] (inverse of unpack_int4; synthetic checkpoints)."""
    out, cols = codes.shape
    u = torch.nn.functional.pad(codes.long() + 8, (0, (-cols) % 8)).reshape(out, -1, 8)
    word = (u << torch.arange(0, 32, 4, dtype=torch.int64)).sum(-1)
    return torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)


def dequant_int4(packed: torch.Tensor, scale: torch.Tensor, cols: int) -> torch.Tensor:
    q = unpack_int4(packed, cols).float()
    return q * scale.float().repeat_interleave(GROUP_INT4, dim=1)[:, :cols]


# ------------------------------------------------------------------------------------------------ E2M1 helpers
def _e2m1_round(y: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 value of y (ties to even, saturating at +-6)."""
    lv = _LEVELS.to(y.device)[F._e2m1_mag_even(y.abs())]
    return torch.copysign(lv, y)


def _e2m1_codes(y: torch.Tensor) -> torch.Tensor:
    mag = F._e2m1_mag_even(y.abs())
    return mag | (((y < 0) & (mag > 0)).int() << 3)


def _best_scale(blocks: torch.Tensor, cands: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
    """blocks [R, nb, B], candidate scales [R, nb, C] (> 0) with a validity mask -> chosen scale [R, nb]: the least
    squared reconstruction error, the first (smallest) candidate on ties."""
    x = blocks[..., None, :]                                             # [R, nb, 1, B]
    s = cands[..., None]                                                 # [R, nb, C, 1]
    err = ((_e2m1_round(x / s) * s - x) ** 2).sum(-1)                    # [R, nb, C]
    err = torch.where(valid, err, torch.full_like(err, float("inf")))
    return cands.gather(-1, err.argmin(-1, keepdim=True)).squeeze(-1)


def _chunked(w: torch.Tensor, fn) -> list:
    return [fn(w[r:r + ROW_CHUNK]) for r in range(0, w.shape[0], ROW_CHUNK)]


# ------------------------------------------------------------------------------------------------ NVFP4
_E4M3_POS = torch.arange(0, 0x7F, dtype=torch.uint8)                    # every finite non-negative E4M3 code byte


def _e4m3_values(device) -> torch.Tensor:
    return _E4M3_POS.view(torch.float8_e4m3fn).float().to(device)


def quant_nvfp4(w: torch.Tensor, search: bool = True, global_scale: Optional[float] = None):
    """fp32 [out, in] -> (weight uint8 [out, in/2], weight_scale E4M3 [out, in/16], weight_scale_2 fp32 [])."""
    out, cols = w.shape
    w = w.float()
    g = float(global_scale) if global_scale else float(w.abs().max()) / (E2M1_MAX * E4M3_MAX)
    g = max(g, 1e-12)
    table = _e4m3_values(w.device)                                      # ascending with the code byte

    def one(rows: torch.Tensor):
        blocks = rows.reshape(rows.shape[0], cols // 16, 16)
        amax = blocks.abs().amax(-1)
        if search:
            lo = torch.searchsorted(table, (amax * WINDOW[0] / g).contiguous())            # first code >= lo
            hi = torch.searchsorted(table, (amax * WINDOW[1] / g).contiguous(), right=True)  # past last code <= hi
            span = 10                                                   # a factor-of-two window holds <= 9 codes
            idx = lo[..., None] + torch.arange(span, device=w.device)
            valid = (idx < hi[..., None]) & (idx >= 1) & (idx < table.numel())
            # empty windows (all-zero blocks, or windows past the E4M3 range) fall back to the nearest code
            near = _nearest_code(table, amax / E2M1_MAX / g)
            none = ~valid.any(-1)
            idx = torch.where(none[..., None], near[..., None].expand_as(idx), idx)
            valid = valid | (none[..., None] & (torch.arange(span, device=w.device) == 0))
            cand = table[idx.clamp(0, table.numel() - 1)] * g
            cand = torch.where(cand > 0, cand, torch.full_like(cand, g))
            sc = _best_scale(blocks, cand, valid)
        else:
            sc = table[_nearest_code(table, amax / E2M1_MAX / g)] * g
            sc = torch.where(sc > 0, sc, torch.full_like(sc, g))
        codes = _e2m1_codes(blocks / sc[..., None]).reshape(rows.shape[0], cols)
        return F.pack_nibbles(codes), (sc / g).to(torch.float8_e4m3fn)
    parts = _chunked(w, one)
    return (torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts]),
            torch.tensor(g, dtype=torch.float32))


def _nearest_code(table: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    i = torch.searchsorted(table, v.contiguous()).clamp(1, table.numel() - 1)
    below = (v - table[i - 1]).abs() <= (table[i] - v).abs()
    return torch.where(below, i - 1, i)


def dequant_nvfp4(weight: torch.Tensor, weight_scale: torch.Tensor, weight_scale_2: torch.Tensor) -> torch.Tensor:
    vals = F.e2m1_decode(F.unpack_nibbles(weight))
    return vals * (weight_scale.float() * float(weight_scale_2)).repeat_interleave(16, dim=1)


# ------------------------------------------------------------------------------------------------ MXFP4
def quant_mxfp4(w: torch.Tensor, search: bool = True):
    """fp32 [out, in] -> (weight uint8 [out, in/2], weight_scale E8M0 uint8 [out, in/32])."""
    out, cols = w.shape
    w = w.float()

    def one(rows: torch.Tensor):
        blocks = rows.reshape(rows.shape[0], cols // 32, 32)
        amax = blocks.abs().amax(-1).clamp(min=2.0 ** -126)
        if search:
            e_lo = torch.ceil(torch.log2(amax * WINDOW_MX[0]))          # powers of two inside the window
            e_hi = torch.floor(torch.log2(amax * WINDOW_MX[1]))
            exps = e_lo[..., None] + torch.arange(3, device=w.device)
            valid = exps <= e_hi[..., None]
            sc = _best_scale(blocks, torch.exp2(exps), valid)
        else:
            sc = torch.exp2(torch.ceil(torch.log2(amax / E2M1_MAX)))  # the smallest power of two without clipping
        e8 = (torch.log2(sc).round() + 127).clamp(0, 254)
        sc = torch.exp2(e8 - 127)
        codes = _e2m1_codes(blocks / sc[..., None]).reshape(rows.shape[0], cols)
        return F.pack_nibbles(codes), e8.to(torch.uint8)
    parts = _chunked(w, one)
    return torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])


def dequant_mxfp4(weight: torch.Tensor, weight_scale: torch.Tensor) -> torch.Tensor:
    vals = F.e2m1_decode(F.unpack_nibbles(weight))
    return vals * torch.exp2(weight_scale.float() - 127.0).repeat_interleave(32, dim=1)


# ------------------------------------------------------------------------------------------------ report
def _sqnr_db(signal: torch.Tensor, noise: torch.Tensor) -> float:
    n = float((noise.double() ** 2).sum())
    return float("inf") if n == 0 else 10.0 * math.log10(float((signal.double() ** 2).sum()) / n)


def report(ref: torch.Tensor, approx: torch.Tensor, probes: int = 128) -> dict:
    """Quality of a converted tensor against its INT4 reference: SQNR in weight space and in output space (a fixed
    batch of +-1 probe activations), largest absolute error, fraction of weights reproduced exactly."""
    d = approx - ref
    g = torch.Generator().manual_seed(1234)
    x = (torch.randint(0, 2, (probes, ref.shape[1]), generator=g).float() * 2 - 1).to(ref.device)
    return {"sqnr_db": round(_sqnr_db(ref, d), 3), "out_sqnr_db": round(_sqnr_db(x @ ref.T, x @ d.T), 3),
            "max_abs_err": float(d.abs().max()), "exact_frac": float((d == 0).float().mean())}


# ------------------------------------------------------------------------------------------------ checkpoints
def _int4_tensors(names) -> dict:
    """prefix -> {"packed", "scale", "shape"} tensor names of every complete INT4 weight in a shard."""
    found: dict = {}
    for n in names:
        for suffix, role in ((".weight_packed", "packed"), (".weight_scale", "scale"), (".weight_shape", "shape")):
            if n.endswith(suffix):
                found.setdefault(n[: -len(suffix)], {})[role] = n
    return {p: r for p, r in found.items() if len(r) == 3}


def convert_tensor(ref: torch.Tensor, fmt: str, search: bool = True) -> tuple[dict, torch.Tensor]:
    """One fp32 weight -> ({suffix: tensor} in the output format, its dequantized value)."""
    if fmt == "nvfp4":
        q, s8, g2 = quant_nvfp4(ref, search)
        return {".weight": q, ".weight_scale": s8, ".weight_scale_2": g2.reshape(1)}, dequant_nvfp4(q, s8, g2)
    if fmt == "mxfp4":
        q, e8 = quant_mxfp4(ref, search)
        return {".weight": q, ".weight_scale": e8}, dequant_mxfp4(q, e8)
    raise ValueError(f"unknown format {fmt!r}")


def convert_file(src: str, dst: str, fmt: str, search: bool = True, input_scales: Optional[dict] = None) -> dict:
    """Convert every INT4 weight of one safetensors shard; every other tensor is copied as is.  -> report per weight."""
    from ..models.loader import SafeTensors, save
    st = SafeTensors(src)
    names = list(st.keys())
    groups = _int4_tensors(names)
    consumed = {n for roles in groups.values() for n in roles.values()}
    out = {n: st.get(n) for n in names if n not in consumed}
    rep = {}
    for prefix, roles in sorted(groups.items()):
        rows, cols = (int(v) for v in st.get(roles["shape"]).tolist())
        ref = dequant_int4(st.get(roles["packed"]), st.get(roles["scale"]), cols)[:rows]
        tensors, approx = convert_tensor(ref, fmt, search)
        for suffix, t in tensors.items():
            out[prefix + suffix] = t
        if fmt == "nvfp4" and input_scales and prefix in input_scales:
            out[prefix + ".input_scale"] = input_scales[prefix].reshape(1).float()
        rep[prefix] = report(ref, approx)
    save(out, dst)
    return rep


def convert(src_dir: str, dst_dir: str, fmt: str, search: bool = True) -> dict:
    """Convert a checkpoint directory one shard at a time (one shard in memory) and write conversion_report.json."""
    os.makedirs(dst_dir, exist_ok=True)
    rep: dict = {}
    for name in sorted(f for f in os.listdir(src_dir) if f.endswith(".safetensors")):
        rep.update(convert_file(os.path.join(src_dir, name), os.path.join(dst_dir, name), fmt, search))
    worst = min((r["sqnr_db"] for r in rep.values()), default=float("inf"))
    with open(os.path.join(dst_dir, "conversion_report.json"), "w") as fh:
        json.dump({"format": fmt, "scale_search": search, "worst_sqnr_db": worst, "tensors": rep}, fh, indent=1)
    return rep


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("convert")
    c.add_argument("--src", required=True)
    c.add_argument("--dst", required=True)
    c.add_argument("--fmt", choices=["nvfp4", "mxfp4"], default="nvfp4")
    c.add_argument("--no-search", action="store_true", help="nominal scale (amax / 6, nearest storable) only")
    a = ap.parse_args()
    rep = convert(a.src, a.dst, a.fmt, not a.no_search)
    print(json.dumps({"tensors": len(rep), "worst_sqnr_db": min((r["sqnr_db"] for r in rep.values()),
                                                                default=None)}))


if __name__ == "__main__":
    main()
