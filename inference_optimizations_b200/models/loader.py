"""HF safetensors checkpoints: a self-contained reader / writer of the safetensors container (8-byte little-endian
header length, JSON header {name: {dtype, shape, data_offsets}}, raw little-endian data) and the tensor-parallel
sharding of Gemma-3 style checkpoints into `GQAModel(weights=...)`.

Sharding (column-parallel q/k/v/gate/up by output rows, row-parallel o/down by input columns) matches
`models/gqa.py`; norms and the tied embedding are replicated (the LM head takes its vocab shard of it).  Reads are memory-mapped, so a rank touches only the
bytes of its own shards."""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Iterable, Optional

import torch

_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "F8_E4M3": torch.float8_e4m3fn,
           "I32": torch.int32, "I64": torch.int64, "U8": torch.uint8, "I8": torch.int8}
_NAMES = {v: k for k, v in _DTYPES.items()}


def read_header(path: str) -> tuple[dict, int]:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
    hdr.pop("__metadata__", None)
    return hdr, 8 + n


class SafeTensors:
    """Lazy, memory-mapped view of one .safetensors file."""

    def __init__(self, path: str):
        self.path = path
        self.header, self.base = read_header(path)
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)

    def keys(self) -> Iterable[str]:
        return self.header.keys()

    def get(self, name: str) -> torch.Tensor:
        meta = self.header[name]
        dt = _DTYPES[meta["dtype"]]
        a, b = meta["data_offsets"]
        buf = self._mm[self.base + a:self.base + b]
        t = torch.frombuffer(bytearray(buf), dtype=torch.uint8)
        return t.view(dt).reshape(meta["shape"]) if meta["shape"] else t.view(dt).reshape(())

    def close(self) -> None:
        self._mm.close()
        self._f.close()


def save(tensors: dict, path: str, metadata: Optional[dict] = None) -> None:
    hdr, off, blobs = {}, 0, []
    for k, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        hdr[k] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    if metadata:
        hdr["__metadata__"] = metadata
    h = json.dumps(hdr).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def open_checkpoint(path: str) -> dict:
    """name -> SafeTensors for a file or a directory of *.safetensors."""
    files = [path] if os.path.isfile(path) else sorted(os.path.join(path, f) for f in os.listdir(path)
                                                       if f.endswith(".safetensors"))
    index = {}
    for fp in files:
        st = SafeTensors(fp)
        for k in st.keys():
            index[k] = st
    return index


def shard_gqa(index: dict, cfg, tp_rank: int, tp: int, device, draft: bool = False) -> dict:
    """HF-named tensors of this rank's shards (bf16 on `device`) for GQAModel(weights=...)."""
    out = {}

    def get(name):
        return index[name].get(name).to(torch.bfloat16)

    def rows(name):          # column-parallel: split output rows
        t = get(name)
        n = t.shape[0] // tp
        return t[tp_rank * n:(tp_rank + 1) * n]

    def cols(name):          # row-parallel: split input columns
        t = get(name)
        n = t.shape[1] // tp
        return t[:, tp_rank * n:(tp_rank + 1) * n]

    n_layers = cfg.draft_layers if draft else cfg.num_layers
    if not draft:   # replicated: the input lookup needs every row; the tied LM head slices its vocab shard
        out["model.embed_tokens.weight"] = get("model.embed_tokens.weight")
    out["model.norm.weight"] = get("model.norm.weight")
    if draft and "fc.weight" in index:
        out["fc.weight"] = get("fc.weight")
    for i in range(n_layers):
        p = f"model.layers.{i}."
        for n in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                  "mlp.gate_proj.weight", "mlp.up_proj.weight"):
            out[p + n] = rows(p + n)
        for n in ("self_attn.o_proj.weight", "mlp.down_proj.weight"):
            out[p + n] = cols(p + n)
        for n in ("self_attn.q_norm.weight", "self_attn.k_norm.weight", "input_layernorm.weight",
                  "post_attention_layernorm.weight", "pre_feedforward_layernorm.weight",
                  "post_feedforward_layernorm.weight"):
            out[p + n] = get(p + n)
    return {k: v.to(device) for k, v in out.items()}


def export_gqa(model, path: str) -> None:
    """Write a tp = 1 GQAModel as an HF-named safetensors file (round-trip tests, handing weights to other tools)."""
    t = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.final_norm}
    for i, (l, g) in enumerate(zip(model.layers, model.geoms)):
        p = f"model.layers.{i}."
        qd, kd = g.q_heads * g.head_dim, g.kv_heads * g.head_dim
        t[p + "self_attn.q_proj.weight"] = l.qkv[:qd]
        t[p + "self_attn.k_proj.weight"] = l.qkv[qd:qd + kd]
        t[p + "self_attn.v_proj.weight"] = l.qkv[qd + kd:]
        t[p + "self_attn.o_proj.weight"] = l.o
        f = l.gu.shape[0] // 2
        t[p + "mlp.gate_proj.weight"] = l.gu[:f]
        t[p + "mlp.up_proj.weight"] = l.gu[f:]
        t[p + "mlp.down_proj.weight"] = l.down
        for n, v in (("self_attn.q_norm.weight", l.q_norm), ("self_attn.k_norm.weight", l.k_norm),
                     ("input_layernorm.weight", l.n_in), ("post_attention_layernorm.weight", l.n_post_attn),
                     ("pre_feedforward_layernorm.weight", l.n_pre_ffn),
                     ("post_feedforward_layernorm.weight", l.n_post_ffn)):
            t[p + n] = v
    save(t, path)
