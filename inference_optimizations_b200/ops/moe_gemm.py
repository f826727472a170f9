"""FP8 block-scaled expert GEMMs (DeepSeek-V3 recipe: E4M3 weights with one power-of-two scale per 128 x 128 block,
E4M3 activations with one per 1 x 128 block) and the fused MoE feed-forward built on them.

Layouts (the kernel contract of `csrc/moe_gemm.cu`):
  * activation rows: uint8 E4M3 [rows, K] + int32 scale words [rows, K / 128], each word the UE8M0 exponent byte
    replicated four times (one byte per 32-wide MMA sub-block);
  * packed weights: per (expert, 128-row tile, 128-wide K chunk) G tiles of 128 x 128 bytes in the SW128 K-major
    layout (16-byte chunk c of row r stored at chunk c ^ (r % 8)), then G scale atoms of 512 bytes (row r = r0 +
    32 r1 at byte 16 r0 + 4 r1 + j).  G = 2 interleaves gate and up rows of the same 128 FFN columns.

Scale rule (`moe-gemm/norm-quant-fused/pro_norm_quant.py:1-17`, UE8M0 form): s = 2^ceil(log2(amax / 448)), q =
e4m3(x / s); computed exactly from the float bits so kernel and oracle agree.

NVFP4 experts (W4A4, the GLM-5 / Kimi serving format; `moe-gemm/w4a4-moe-decode-gemm/moe_decode_gemm.py:1-25`,
`moe-gemm/cutedsl-grouped-nvfp4/nvfp4_layout.py:1-20`): weights E2M1 with one E4M3 scale per 16 values and one fp32
global scale per expert (gate and up share it), activations E2M1 + E4M3 per 16 (global 1).  Same 128-byte K chunks
(256 values), four scale atoms per tile per chunk (MMA j of K = 64 reads atom j).
"""
from __future__ import annotations

import torch
import torch.nn.functional as Fn

from typing import Optional

from .._ext import ext
from . import formats as FM

TILE = 128
INV448 = torch.tensor(1.0 / 448.0, dtype=torch.float32)


def ue8m0_exponent(amax: torch.Tensor) -> torch.Tensor:
    """Biased UE8M0 byte (int32) of the smallest power of two s with amax / s <= 448, clamped to [1, 253]."""
    x = amax.float() * INV448.to(amax.device)
    bits = x.view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).int()
    e = torch.where(x == 0, torch.full_like(e, -126), e)
    return e.clamp(-126, 126) + 127


def _pow2(eb: torch.Tensor) -> torch.Tensor:
    return torch.exp2(eb.float() - 127.0)


def quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [R, K] (K % 128 == 0) -> (q uint8 [R, K], scale words int32 [R, K / 128])."""
    r, k = x.shape
    g = x.float().view(r, k // TILE, TILE)
    eb = ue8m0_exponent(g.abs().amax(-1))
    q = (g / _pow2(eb)[..., None]).to(torch.float8_e4m3fn).view(torch.uint8).view(r, k)
    return q, (eb * 0x01010101).to(torch.int32)


def dequant_rows(q: torch.Tensor, sc: torch.Tensor) -> torch.Tensor:
    r, k = q.shape
    v = q.view(torch.float8_e4m3fn).float().view(r, k // TILE, TILE)
    return (v * _pow2(sc & 0xFF)[..., None]).view(r, k)


def quant_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [..., N, K] -> (q uint8 [..., N, K], exponent bytes uint8 [..., N / 128, K / 128])."""
    *lead, n, k = w.shape
    b = w.float().reshape(*lead, n // TILE, TILE, k // TILE, TILE)
    eb = ue8m0_exponent(b.abs().amax(dim=(-3, -1)))
    q = (b / _pow2(eb)[..., :, None, :, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    return q.reshape(*lead, n, k), eb.to(torch.uint8)


def _quant_blocks_per_expert(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quant_blocks one expert at a time: the fp32 temporaries stay one expert large (weight preparation of big
    expert sets must not need several times the weights in scratch memory)."""
    qs, es = zip(*(quant_blocks(w[e]) for e in range(w.shape[0])))
    return torch.stack(qs), torch.stack(es)


def dequant_blocks(q: torch.Tensor, eb: torch.Tensor) -> torch.Tensor:
    *lead, n, k = q.shape
    v = q.view(torch.float8_e4m3fn).float().reshape(*lead, n // TILE, TILE, k // TILE, TILE)
    return (v * _pow2(eb.int())[..., :, None, :, None]).reshape(*lead, n, k)


def _sw128(tiles: torch.Tensor) -> torch.Tensor:
    """[..., 128, 128] bytes -> SW128 order (16-byte chunk c of row r at chunk c ^ (r % 8))."""
    r = torch.arange(TILE, device=tiles.device)
    idx = (torch.arange(8, device=tiles.device)[None, :] ^ (r[:, None] % 8))          # out[r, j] = in[r, j ^ r%8]
    t = tiles.reshape(*tiles.shape[:-1], 8, 16)
    idx = idx.view(*([1] * (t.dim() - 3)), TILE, 8, 1).expand(*t.shape[:-3], TILE, 8, 16)
    return torch.gather(t, -2, idx).reshape(tiles.shape)


def sf_atom(eb_rows: torch.Tensor) -> torch.Tensor:
    """Scale bytes of 128 rows -> the 512-byte scale atom (row r0 + 32 r1 at 16 r0 + 4 r1 + j, j < 4).  eb_rows is
    [..., 128] (one byte per row, replicated over j) or [..., 128, 4] (byte j of each row)."""
    if eb_rows.shape[-1] != 4 or eb_rows.dim() == 1:
        eb_rows = eb_rows[..., None].expand(*eb_rows.shape, 4)
    lead = eb_rows.shape[:-2]
    v = eb_rows.reshape(*lead, 4, 32, 4)                            # [.., r1, r0, j]
    return v.transpose(-2, -3).reshape(*lead, 512)


def pack_weights(qs: list, ebs: list) -> torch.Tensor:
    """Pack G quantized weights that feed the same CTA (each q [E, N, K] uint8 with exponent bytes eb either per
    128 x 128 block [E, N/128, K/128] or per row and 128-chunk [E, N, K/128]) into
    [E, N/128, K/128, G * (16384 + 512)] uint8."""
    E, N, K = qs[0].shape
    nt, kc = N // TILE, K // TILE
    tiles, atoms = [], []
    for q, eb in zip(qs, ebs):
        t = q.view(E, nt, TILE, kc, TILE).permute(0, 1, 3, 2, 4).contiguous()             # [E, nt, kc, 128, 128]
        tiles.append(_sw128(t).reshape(E, nt, kc, TILE * TILE))
        if eb.shape[1] == nt:                                                              # block scale: all rows
            atoms.append(eb.view(E, nt, kc, 1).expand(E, nt, kc, 512))
        else:
            rows = eb.view(E, nt, TILE, kc).permute(0, 1, 3, 2)                            # [E, nt, kc, 128]
            atoms.append(sf_atom(rows))
    return torch.cat(tiles + atoms, dim=-1).contiguous()


def pack_weights_paired(q: torch.Tensor, eb: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Plain-output weights: when N % 256 == 0 pack output tiles 2j and 2j + 1 into one block (one CTA computes
    256 output columns per item: half the items and weight-tile issue overhead).  Returns (packed, G)."""
    E, N, K = q.shape
    if N % 256:
        return pack_weights([q], [eb]), 1
    qv = q.view(E, N // 256, 2, TILE, K)
    per_row = eb.shape[1] == N
    ev = eb.view(E, N // 256, 2, TILE, -1) if per_row else eb.view(E, N // 256, 2, -1)
    qs = [qv[:, :, g].reshape(E, N // 2, K) for g in range(2)]
    es = [ev[:, :, g].reshape(E, N // 2, -1) if per_row else ev[:, :, g] for g in range(2)]
    return pack_weights(qs, es), 2


def quant_nvfp4_weights(w: torch.Tensor, groups: int = 1) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """w [E, N, K] -> (E2M1 pairs uint8 [E, N, K/2], E4M3 scale bytes uint8 [E, N, K/16], global fp32 [E]); the
    global scale is amax / (448 * 6) over each expert (over `groups` consecutive N-blocks jointly when gate and up
    are stacked: pass them concatenated along N with groups = 1)."""
    E, N, K = w.shape
    qs, ss, gs = [], [], []
    for e in range(E):
        g = max(float(w[e].abs().amax()) / (448.0 * 6.0), 1e-30)
        q, s8 = FM.nvfp4_quantize(w[e].float(), g)
        qs.append(q)
        ss.append(s8.view(torch.uint8))
        gs.append(g)
    return torch.stack(qs), torch.stack(ss), torch.tensor(gs, dtype=torch.float32, device=w.device)


def dequant_nvfp4_weights(q: torch.Tensor, s8: torch.Tensor, gs: torch.Tensor) -> torch.Tensor:
    return torch.stack([FM.nvfp4_dequantize(q[e], s8[e].view(torch.float8_e4m3fn), float(gs[e]))
                        for e in range(q.shape[0])])


def quant_nvfp4_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [R, K] -> (E2M1 pairs uint8 [R, K/2], E4M3 scale bytes as int32 words [R, K/64]) with global scale 1."""
    q, s8 = FM.nvfp4_quantize(x.float(), 1.0)
    return q, s8.view(torch.uint8).contiguous().view(torch.int32)


def dequant_nvfp4_rows(q: torch.Tensor, sc: torch.Tensor) -> torch.Tensor:
    return FM.nvfp4_dequantize(q, sc.contiguous().view(torch.uint8).view(torch.float8_e4m3fn), 1.0)


def pack_weights_nvfp4(qs: list, scs: list) -> torch.Tensor:
    """Pack G NVFP4 weights (each E2M1 pairs [E, N, K/2], scale bytes [E, N, K/16]) into
    [E, N/128, K/256, G * (16384 + 4 * 512)] uint8: G SW128 tiles, then atoms [g][j] (MMA j of the chunk)."""
    E, N, Kh = qs[0].shape
    nt, kc = N // TILE, Kh // TILE
    tiles, atoms = [], []
    for q in qs:
        t = q.reshape(E, nt, TILE, kc, TILE).permute(0, 1, 3, 2, 4).contiguous()
        tiles.append(_sw128(t).reshape(E, nt, kc, TILE * TILE))
    for sc in scs:
        v = sc.reshape(E, nt, TILE, kc, 4, 4).permute(0, 1, 3, 4, 2, 5)                  # [E, nt, kc, j, 128, 4]
        atoms.append(sf_atom(v).reshape(E, nt, kc, 4 * 512))
    return torch.cat(tiles + atoms, dim=-1).contiguous()


def gemm(wpack, x, x_scale, off, pairs, out, status, *, n_tiles: int, kc: int, g: int, nt: int, mode: int,
         src_div: int, src_limit: int = 1 << 30, src_shared_base: int = 0, pair_w=None, out_scale=None, out_mul: float = 1.0,
         num_ctas: int = 148, kind: int = 0, expert_mul=None, out_peers=None, out_offset: int = 0, out_div: int = 1,
         out_rank: int = 0, out_shared_base: int = 0, pairs_total: int = 0, ksplit: int = 1,
         split_rows: int = 0, src_group: int = 0, src_group_stride: int = 0, static_index: bool = False,
         red_out=None, tile_cnt=None, out_bcast: int = 0) -> None:
    """One grouped block-scaled GEMM launch (argument meanings: `MoeGemmArgs` in csrc/kernels.h).  Launched with
    programmatic dependent launch unless `PDL` is off: the kernel sets up (and, with `static_index` -- off / pairs
    complete before the previous kernel ran -- starts streaming weights) while the previous kernel finishes.  When
    `TRACE` holds an int64 CUDA tensor, CTA 0's phase timeline (clock64, `MgTraceEv` order) is written into it."""
    ext().moe_gemm(wpack, x, x_scale, off, pairs, pair_w, out, out_scale, status, n_tiles, kc, g, nt, mode, src_div,
                   src_limit, src_shared_base, out_mul, num_ctas, kind, expert_mul, out_peers, out_offset, out_div, out_rank,
                   out_shared_base, pairs_total, ksplit, split_rows, src_group, src_group_stride, TRACE[0], PDL[0],
                   static_index, red_out, tile_cnt, out_bcast)


TRACE: list = [None]
PDL: list = [True]
# Which set of cached scratch buffers (split-K partials, per-step workspaces) the launches use: 0 by default, 1 while
# the split-prefill lane enqueues its layers (`engine/pdmux.py`) -- that lane runs concurrently with decode on another
# stream, so the two must never share a scratch buffer of the same shape.
LANE: list = [0]


def static_index_tensors(make) -> tuple:
    """Index tensors for a GEMM whose work list never changes (dense linears, head-batched products): built by
    `make()` and, outside stream capture, completed before returning, so launches may read them before waiting on the
    previous kernel.  -> (tensors..., complete flag)."""
    t = make()
    done = False
    if torch.cuda.is_available() and t[0].is_cuda and not torch.cuda.is_current_stream_capturing():
        torch.cuda.current_stream(t[0].device).synchronize()
        done = True
    return (*t, done)


_TACTICS = None


def _tactics() -> dict:
    """Measured token-tile choice per routed-token count (`moe_tactics.json` next to this file, written by
    `utils/microbench.py moe_tactics`): the per-token-count tactic table idea of
    `moe-gemm/moe-tactic-tables/numinous_moe_tactics.py:1-25`, lookup = the smallest measured count >= n."""
    global _TACTICS
    if _TACTICS is None:
        import json
        import os
        p = os.path.join(os.path.dirname(__file__), "moe_tactics.json")
        _TACTICS = {}
        if os.path.exists(p):
            with open(p) as f:
                _TACTICS = json.load(f)
    return _TACTICS


def tactic_nt(tokens: int, fmt: str = "fp8") -> Optional[int]:
    table = _tactics().get(fmt)
    if not table:
        return None
    keys = sorted(int(k) for k in table)
    for k in keys:
        if k >= tokens:
            return int(table[str(k)])
    return int(table[str(keys[-1])])


def pick_nt(rows_per_expert: int) -> int:
    """Token tile (the MMA's N) for an expected number of rows per expert."""
    for nt in (16, 32, 64):
        if rows_per_expert <= nt:
            return nt
    return 128


class BlockScaledExperts:
    """Routed (+ one shared) SwiGLU experts with block-scaled weights (fmt "fp8": E4M3 + UE8M0 per 128 x 128;
    "nvfp4": E2M1 + E4M3 per 16 + fp32 per expert), executed by two grouped GEMM launches: gate/up with fused
    SwiGLU + re-quantization (to the same format), then down with the routing weight folded into the epilogue; a
    combine kernel sums each token's top-k rows (+ shared) in slot order."""

    def __init__(self, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
                 shared: tuple | None = None, fmt: str = "fp8", num_ctas: int | None = None):
        """w_gate / w_up [E, F, H], w_down [E, H, F] (any float dtype, quantized here one expert at a time);
        shared = (g, u, d) of one expert with the same shapes minus E."""
        if shared is not None:
            w_gate = torch.cat([w_gate, shared[0][None]])
            w_up = torch.cat([w_up, shared[1][None]])
            w_down = torch.cat([w_down, shared[2][None]])
        self.fmt, self.kind = fmt, {"fp8": 0, "nvfp4": 1}[fmt]
        self.has_shared = shared is not None
        self.E = w_gate.shape[0] - int(self.has_shared)
        self.F, self.H = w_gate.shape[1], w_gate.shape[2]
        dev = w_gate.device
        if fmt == "fp8":
            qg, eg = _quant_blocks_per_expert(w_gate)
            qu, eu = _quant_blocks_per_expert(w_up)
            qd, ed = _quant_blocks_per_expert(w_down)
            self.q = (qg, eg, qu, eu, qd, ed)
            self.w1 = pack_weights([qg, qu], [eg, eu])
            self.w2, self.g2 = pack_weights_paired(qd, ed)
            self.mul1 = self.mul2 = None
        else:
            qgu, sgu, ggu = quant_nvfp4_weights(torch.cat([w_gate, w_up], dim=1))   # gate and up share a global
            qd, sd, gd = quant_nvfp4_weights(w_down)
            F = self.F
            self.q = (qgu, sgu, ggu, qd, sd, gd)
            self.w1 = pack_weights_nvfp4([qgu[:, :F], qgu[:, F:]], [sgu[:, :F], sgu[:, F:]])
            self.w2 = pack_weights_nvfp4([qd], [sd])
            self.g2 = 1
            self.mul1, self.mul2 = ggu, gd
        self.num_ctas = num_ctas or (torch.cuda.get_device_properties(dev).multi_processor_count
                                     if dev.type == "cuda" else 1)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._parts: dict = {}

    @classmethod
    def build(cls, e_lo: int, e_hi: int, F: int, H: int, gen, shared: tuple | None = None, fmt: str = "fp8",
              device=None) -> "BlockScaledExperts":
        """Experts e_lo .. e_hi - 1 from gen(e) -> (w_gate [F, H], w_up [F, H], w_down [H, F]), quantized and packed
        one expert at a time straight into the launch layout: no stacked bf16 or fp32 copy of the expert set ever
        exists, so a node-size expert set is built in the memory its packed form needs.  Same packed bytes as the
        stacked constructor (quantization is per expert in both).  No dequantization oracle is kept."""
        self = cls.__new__(cls)
        self.fmt, self.kind = fmt, {"fp8": 0, "nvfp4": 1}[fmt]
        self.has_shared = shared is not None
        self.E, self.F, self.H = e_hi - e_lo, F, H
        n = self.E + int(self.has_shared)
        dev = device or (shared[0].device if shared is not None else gen(e_lo)[0].device)
        self.q = None
        if self.kind == 0:
            self.g2 = 2 if H % 256 == 0 else 1
            self.w1 = torch.empty(n, F // TILE, H // TILE, 2 * (16384 + 512), dtype=torch.uint8, device=dev)
            self.w2 = torch.empty(n, H // (TILE * self.g2), F // TILE, self.g2 * (16384 + 512), dtype=torch.uint8,
                                  device=dev)
            self.mul1 = self.mul2 = None
        else:
            self.g2 = 1
            self.w1 = torch.empty(n, F // TILE, H // (2 * TILE), 2 * (16384 + 4 * 512), dtype=torch.uint8, device=dev)
            self.w2 = torch.empty(n, H // TILE, F // (2 * TILE), 16384 + 4 * 512, dtype=torch.uint8, device=dev)
            self.mul1 = torch.empty(n, dtype=torch.float32, device=dev)
            self.mul2 = torch.empty(n, dtype=torch.float32, device=dev)
        for j in range(n):
            g, u, d = shared if j == self.E else gen(e_lo + j)
            if self.kind == 0:
                qg, eg = quant_blocks(g[None])
                qu, eu = quant_blocks(u[None])
                self.w1[j] = pack_weights([qg, qu], [eg, eu])[0]
                del qg, qu
                qd, ed = quant_blocks(d[None])
                self.w2[j] = pack_weights_paired(qd, ed)[0][0]
            else:
                qgu, sgu, ggu = quant_nvfp4_weights(torch.cat([g, u])[None])
                self.w1[j] = pack_weights_nvfp4([qgu[:, :F], qgu[:, F:]], [sgu[:, :F], sgu[:, F:]])[0]
                qd, sd, gd = quant_nvfp4_weights(d[None])
                self.w2[j] = pack_weights_nvfp4([qd], [sd])[0]
                self.mul1[j], self.mul2[j] = ggu[0], gd[0]
            del g, u, d
        self.num_ctas = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 1
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._parts: dict = {}
        return self

    @classmethod
    def random_packed(cls, E: int, F: int, H: int, fmt: str = "fp8", shared: bool = True, device="cuda",
                      seed: int = 0) -> "BlockScaledExperts":
        """Experts with random packed weights straight in the kernel layout (no bf16 master copy: benchmark-size
        expert sets fit on the device).  Values are finite E4M3 / E2M1 codes with moderate scales."""
        self = cls.__new__(cls)
        self.fmt, self.kind = fmt, {"fp8": 0, "nvfp4": 1}[fmt]
        self.has_shared, self.E, self.F, self.H = shared, E, F, H
        n = E + int(shared)
        g = torch.Generator(device=device).manual_seed(seed)
        sfw, vals = (1, TILE) if self.kind == 0 else (4, 2 * TILE)

        def rand(n_tiles, kc, gg):
            w = torch.randint(0, 256, (n, n_tiles, kc, gg * (16384 + 512 * sfw)), dtype=torch.uint8, device=device,
                              generator=g)
            if self.kind == 0:
                w[(w & 0x7F) == 0x7F] = 0
            w[..., gg * 16384:] = 118 if self.kind == 0 else 0x18            # 2^-9 (UE8M0) / 2^-6 (E4M3)
            return w
        self.g2 = 2 if (self.kind == 0 and H % 256 == 0) else 1
        self.w1 = rand(F // TILE, H // vals, 2)
        self.w2 = rand(H // (TILE * self.g2), F // vals, self.g2)
        self.mul1 = self.mul2 = None
        self.q = None
        self.num_ctas = torch.cuda.get_device_properties(device).multi_processor_count
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._parts = {}
        return self

    def dequant(self):
        if self.fmt == "fp8":
            qg, eg, qu, eu, qd, ed = self.q
            return dequant_blocks(qg, eg), dequant_blocks(qu, eu), dequant_blocks(qd, ed)
        qgu, sgu, ggu, qd, sd, gd = self.q
        gu = dequant_nvfp4_weights(qgu, sgu, ggu)
        return gu[:, :self.F], gu[:, self.F:], dequant_nvfp4_weights(qd, sd, gd)

    def _quant_x(self, x: torch.Tensor):
        t, dev = x.shape[0], x.device
        if self.kind == 0:
            xq = torch.empty(t, self.H, dtype=torch.uint8, device=dev)
            xs = torch.empty(t, self.H // TILE, dtype=torch.int32, device=dev)
        else:
            xq = torch.empty(t, self.H // 2, dtype=torch.uint8, device=dev)
            xs = torch.empty(t, self.H // 64, dtype=torch.int32, device=dev)
        ext().rmsnorm_quant(x.contiguous(), None, 0.0, 0.0, xq, xs, self.kind)
        return xq, xs

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, nt: int | None = None,
                e0: int = 0, xq8: Optional[tuple] = None) -> torch.Tensor:
        """x bf16 [T, H] (already normalized), ids int32 [T, k] (expert ids; this set holds experts e0 .. e0 + E - 1:
        pairs routed to others are not computed and must carry weight 0), w fp32 [T, k] -> bf16 [T, H]."""
        t, k = ids.shape
        dev = x.device
        P = t * k
        extra = t if self.has_shared else 0
        E = self.E + int(self.has_shared)
        # xq8: x already block-quantized by the norm that produced it (FP8 experts only)
        xq, xs = xq8 if (xq8 is not None and self.kind == 0) else self._quant_x(x)
        off = torch.empty(E + 1, dtype=torch.int32, device=dev)
        pairs = torch.empty(P + extra, dtype=torch.int32, device=dev)
        ext().moe_align(ids.contiguous().view(-1), e0, self.E, extra, off, pairs)
        nt = nt or tactic_nt(t, self.fmt) or pick_nt(max(1, -(-2 * P // self.E)))
        kc1 = self.H // (TILE if self.kind == 0 else 2 * TILE)
        kc2 = self.F // (TILE if self.kind == 0 else 2 * TILE)
        if self.kind == 0:
            h = torch.empty(P + extra, self.F, dtype=torch.uint8, device=dev)
            hs = torch.empty(P + extra, self.F // TILE, dtype=torch.int32, device=dev)
        else:
            h = torch.empty(P + extra, self.F // 2, dtype=torch.uint8, device=dev)
            hs = torch.empty(P + extra, self.F // 64, dtype=torch.int32, device=dev)
        gemm(self.w1, xq, xs, off, pairs, h, self.status, n_tiles=self.F // TILE, kc=kc1, g=2, nt=nt, mode=1,
             src_div=k, src_limit=P, out_scale=hs, num_ctas=self.num_ctas, kind=self.kind, expert_mul=self.mul1)
        n2 = self.H // (TILE * self.g2)
        ks = self._dense_split(n2, kc2, nt) if (self.E == 1 and not self.has_shared and k == 1 and t <= 64) else 1
        if ks > 1:
            # a dense FFN at decode sizes: its down projection has only H / 256 output tiles, so K is split and the
            # fp32 partials are summed in split order by one reduction kernel straight into the output (one pair
            # per token, weight 1: no combine).  The split depends on the weight shape only, so every batch of up to
            # 64 tokens rounds the same way (data-parallel ranks agree with one GPU).
            key = (P, ks, LANE[0])
            if key not in self._parts:
                self._parts[key] = torch.empty(ks * P, self.H, dtype=torch.float32, device=dev)
            part = self._parts[key]
            gemm(self.w2, h, hs, off, pairs, part, self.status, n_tiles=n2, kc=kc2, g=self.g2, nt=nt, mode=3,
                 src_div=1, num_ctas=self.num_ctas, kind=self.kind, expert_mul=self.mul2, ksplit=ks, split_rows=P,
                 static_index=True)
            y = torch.empty(t, self.H, dtype=torch.bfloat16, device=dev)
            ext().splitk_reduce(part, ks, y, None, 0, 0, 0)
            return y
        # expert rows stay unweighted in bf16; the combine applies the routing weights in fp32 -- the same rounding
        # points as the expert-parallel exchange (parallel/ep.py), so EP at any width reproduces this path bit for bit.
        # The work list (off / pairs) was complete before the gate/up GEMM passed its dependency wait, so this launch
        # may build it and stream weights while that GEMM finishes.
        rows = torch.empty(P + extra, self.H, dtype=torch.bfloat16, device=dev)
        gemm(self.w2, h, hs, off, pairs, rows, self.status, n_tiles=n2, kc=kc2, g=self.g2,
             nt=nt, mode=0, src_div=1, num_ctas=self.num_ctas, kind=self.kind, expert_mul=self.mul2,
             static_index=True)
        y = torch.empty(t, self.H, dtype=torch.bfloat16, device=dev)
        ext().moe_combine(rows, t, k, P if self.has_shared else -1, w.float().contiguous(), y)
        return y

    def _dense_split(self, n_tiles: int, kc: int, nt: int) -> int:
        """K splits of a dense FFN's down projection at decode sizes (the linear layers' split rule at one token)."""
        from .linear import split_k
        return split_k(n_tiles, 1, nt, kc, self.num_ctas, g=self.g2)

    def forward_ref(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """fp32 oracle of the same arithmetic: quantized activations, quantized SwiGLU output, bf16 rows, fp32
        slot-order sum."""
        wg, wu, wd = (m.to(x.device) for m in self.dequant())
        t, k = ids.shape
        qr, dr = (quant_rows, dequant_rows) if self.kind == 0 else (quant_nvfp4_rows, dequant_nvfp4_rows)
        xd = dr(*qr(x.float()))
        pairs = [(tt, kk, int(ids[tt, kk])) for tt in range(t) for kk in range(k)]
        if self.has_shared:
            pairs += [(tt, -1, self.E) for tt in range(t)]
        out = torch.zeros(t, self.H, dtype=torch.float32, device=x.device)
        for tt, kk, e in pairs:
            hh = Fn.silu(xd[tt] @ wg[e].T) * (xd[tt] @ wu[e].T)
            hd = dr(*qr(hh[None]))[0]
            r = (hd @ wd[e].T) * (float(w[tt, kk]) if kk >= 0 else 1.0)
            out[tt] += r.to(torch.bfloat16).float()
        return out.to(torch.bfloat16)


Fp8Experts = BlockScaledExperts
