"""Dense bf16 linear layers on the weight-streaming tcgen05 GEMM (csrc/moe_gemm.cu, kind::f16 variant).

At decode the token count is small (tens of rows) and a linear layer is a pass over its weights.  The weights are
packed once into UMMA-ready blocks (128 rows x 64 values, SW128, two adjacent 128-row tiles per block when N allows)
so each pipeline stage is one contiguous bulk copy; the tokens are the MMA's N operand (swap-AB), so the weights
stream at full tensor-core width whatever the batch.  y = x W^T exactly like `torch.nn.functional.linear` (fp32
accumulation, bf16 out).  When the output tiles alone cannot occupy every SM (small N, long K: o_proj, down), K is
split into ranges: each (weight tile, token tile, K range) item writes fp32 partials and one kernel sums them in
split order (deterministic) and rounds once.
"""
from __future__ import annotations

import torch

from . import moe_gemm as MG

TILE = 128


def pack_bf16(w: torch.Tensor, g: int) -> torch.Tensor:
    """w bf16 [N, K] -> [1, N / (128 g), K / 64, g * 16384] uint8: g adjacent 128-row tiles per block."""
    N, K = w.shape
    kc = K // 64
    b = w.contiguous().view(torch.uint8).view(N // (TILE * g), g, TILE, kc, 128)     # [nt, g, row, kc, 128 B]
    t = b.permute(0, 3, 1, 2, 4).contiguous()                                         # [nt, kc, g, 128, 128]
    t = MG._sw128(t)
    return t.reshape(1, N // (TILE * g), kc, g * TILE * TILE)


def split_k(n_tiles: int, tokens: int, nt: int, kc: int, ctas: int, min_chunks: int = 4, fill: int = 6,
            red: int = 8, g: int = 1) -> int:
    """K splits for a weight-streaming GEMM with n_tiles output tiles (of 128 g columns): the split count minimizing
    the critical path in units of one CTA's weight chunk (16 KB per 128-column tile):
    waves x (K chunks per split + `fill`, an item's pipeline start) and, when split, + `red` (the reduction launch)
    + the fp32 partials written and read back, spread over the CTAs; each K range at least `min_chunks` chunks; ties
    keep fewer splits.  Measured kernel time at 32 tokens, Gemma-31B bf16 shapes: 64 output tiles (sliding qkv)
    47.9 us unsplit / 35.6 us in 2; 168 tiles (gate_up) 101 us unsplit / 84 us in 2-6; 21 tiles (o) 67.9 us unsplit
    / 22 us in 6-7."""
    items = n_tiles * -(-tokens // nt)
    best, best_cost = 1, None
    for ks in range(1, max(1, kc // min_chunks) + 1):
        cost = -(-items * ks // ctas) * (-(-kc // ks) + fill)
        if ks > 1:
            cost += red + ks * tokens * n_tiles * 128 * g * 8 / (ctas * 16384 * g)
        if best_cost is None or cost < best_cost:
            best, best_cost = ks, cost
    return best


def _splitk_gemm(lin, x, xs, out, t: int, kc: int, kind: int, push=None) -> None:
    """Run lin's GEMM with split-K when it helps: fp32 partials, then one deterministic reduction (to out's dtype:
    bf16, or fp32 for an fp32 `out`).  push = (peers int64 [n], byte offset, n, rank): tensor-parallel push -- the
    kernel writing the final bf16 rows (the GEMM itself, or the split-K reduction) stores each row into this rank's
    slot of all n ranks' symmetric buffers (`out` is the local view of that slot, for the row stride)."""
    from .._ext import ext
    nt = FORCE["nt"] or MG.pick_nt(t)
    n_tiles = lin.N // (TILE * lin.g)
    ks = FORCE["ks"] or split_k(n_tiles, t, nt, kc, lin.num_ctas, g=lin.g)
    off, pairs, static = lin._index(t, x.device)
    f32 = out.dtype == torch.float32
    if push is not None:
        assert not f32 and out.stride(0) == lin.N, "push: bf16 rows of the full width"
    if ks == 1:
        pk = {} if push is None else dict(out_peers=push[0], out_offset=push[1], out_bcast=push[2], out_rank=push[3])
        MG.gemm(lin.wpack, x, xs, off, pairs, out, lin.status, n_tiles=n_tiles, kc=kc, g=lin.g, nt=nt,
                mode=MODE_F32_SPLIT if f32 else 0, src_div=1, num_ctas=lin.num_ctas, kind=kind,
                split_rows=t if f32 else 0, static_index=static, **pk)
        return
    key = (t, ks, MG.LANE[0])
    if key not in lin._parts:
        # fp32 partials and the per-tile counters of the folded reduction (zero between launches: the split that
        # completes a tile re-arms its counter)
        lin._parts[key] = (torch.empty(ks * t, lin.N, dtype=torch.float32, device=x.device),
                           torch.zeros(n_tiles * -(-t // nt), dtype=torch.int32, device=x.device))
    part, cnt = lin._parts[key]
    if FOLD_SPLITK[0] and t <= FOLD_MAX_TOKENS and push is None:
        # few tokens: the split completing a tile reduces it (no reduction launch); with many tokens one CTA's share
        # of the reduction would sit on the critical path, so the separate reduction kernel spreads it instead
        MG.gemm(lin.wpack, x, xs, off, pairs, part, lin.status, n_tiles=n_tiles, kc=kc, g=lin.g, nt=nt,
                mode=MODE_F32_SPLIT, src_div=1, num_ctas=lin.num_ctas, kind=kind, ksplit=ks, split_rows=t,
                static_index=static, red_out=out, tile_cnt=cnt)
        return
    MG.gemm(lin.wpack, x, xs, off, pairs, part, lin.status, n_tiles=n_tiles, kc=kc, g=lin.g, nt=nt,
            mode=MODE_F32_SPLIT, src_div=1, num_ctas=lin.num_ctas, kind=kind, ksplit=ks, split_rows=t,
            static_index=static)
    if push is None:
        ext().splitk_reduce(part, ks, out, None, 0, 0, 0)
    else:
        ext().splitk_reduce(part, ks, out, push[0], push[1], push[2], push[3])


MODE_F32_SPLIT = 3
# tactic overrides for sweeps (utils/microbench.py proj_gemms --nt / --ks); None = the heuristics
FORCE: dict = {"nt": None, "ks": None}
# split-K reduction folded into the GEMM (the split completing a tile reduces it) instead of the separate reduction
# kernel.  Off by default: measured at 8 and 64 decode tokens, the completing split's serial partial sums cost more
# than the separate launch, whose start the programmatic dependent launch already overlaps.
FOLD_SPLITK: list = [False]
FOLD_MAX_TOKENS = 16


class DenseLinear:
    def __init__(self, w: torch.Tensor):
        N, K = w.shape
        assert N % TILE == 0 and K % 64 == 0 and w.dtype == torch.bfloat16
        self.N, self.K = N, K
        self.g = 2 if N % 256 == 0 else 1
        self.wpack = pack_bf16(w, self.g)
        dev = w.device
        self.num_ctas = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 1
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._rows: dict = {}
        self._parts: dict = {}

    def _index(self, t: int, dev):
        if t not in self._rows:
            self._rows[t] = MG.static_index_tensors(lambda: (torch.tensor([0, t], dtype=torch.int32, device=dev),
                                                             torch.arange(t, dtype=torch.int32, device=dev)))
        return self._rows[t]

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, out_f32: bool = False,
                 push=None) -> torch.Tensor:
        """y = x W^T, bf16 out; out_f32: fp32 out (the accumulator as is, no rounding: router logits).  push: a
        push-mode `parallel.symm.TPComm` -- the rows go to this rank's slot of every rank's buffer (the returned
        tensor is the local copy) for the fused all-reduce that follows."""
        t = x.shape[0]
        pk = None
        if push is not None:
            out, *pk = push.push_args(t)
        if out is None:
            out = torch.empty(t, self.N, dtype=torch.float32 if out_f32 else torch.bfloat16, device=x.device)
        if t == 0:
            return out
        xb = x.contiguous().view(torch.uint8)
        _splitk_gemm(self, xb, xb, out, t, self.K // 64, 2, pk)
        return out

    def partials(self, x: torch.Tensor) -> tuple[torch.Tensor, int]:
        """fp32 x W^T left as its split-K partials: ([ks * t, N] split-major, ks), for a consumer that sums the
        splits itself in split order (the router kernel); ks = 1 is the plain fp32 product.  No reduction launch."""
        t = x.shape[0]
        kc = self.K // 64
        nt = FORCE["nt"] or MG.pick_nt(t)
        n_tiles = self.N // (TILE * self.g)
        ks = FORCE["ks"] or split_k(n_tiles, t, nt, kc, self.num_ctas, g=self.g)
        if ks == 1 or t == 0:
            return self(x, out_f32=True), 1
        key = (t, ks, MG.LANE[0])
        if key not in self._parts:
            self._parts[key] = (torch.empty(ks * t, self.N, dtype=torch.float32, device=x.device),
                                torch.zeros(n_tiles * -(-t // nt), dtype=torch.int32, device=x.device))
        part = self._parts[key][0]
        off, pairs, static = self._index(t, x.device)
        xb = x.contiguous().view(torch.uint8)
        MG.gemm(self.wpack, xb, xb, off, pairs, part, self.status, n_tiles=n_tiles, kc=kc, g=self.g, nt=nt,
                mode=MODE_F32_SPLIT, src_div=1, num_ctas=self.num_ctas, kind=2, ksplit=ks, split_rows=t,
                static_index=static)
        return part, ks


class Fp8Linear:
    """y = x W^T with W stored FP8 E4M3 + one UE8M0 scale per 128 x 128 block and x quantized per 1 x 128 on the fly
    (the DeepSeek-V3 FP8 linear; the FP8 LM head of `moe-gemm/fp8-lm-head/pro_fp8_lm_head.py:1-15`), on the grouped
    block-scaled GEMM with one "expert" holding every token."""

    def __init__(self, w: torch.Tensor):
        N, K = w.shape
        assert N % TILE == 0 and K % TILE == 0
        self.N, self.K = N, K
        q, eb = MG.quant_blocks(w[None])
        self.wpack, self.g = MG.pack_weights_paired(q, eb)
        self.q, self.eb = q, eb
        dev = w.device
        self.num_ctas = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 1
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._rows: dict = {}
        self._parts: dict = {}

    def _index(self, t: int, dev):
        if t not in self._rows:
            self._rows[t] = MG.static_index_tensors(lambda: (torch.tensor([0, t], dtype=torch.int32, device=dev),
                                                             torch.arange(t, dtype=torch.int32, device=dev)))
        return self._rows[t]

    def dequant(self) -> torch.Tensor:
        return MG.dequant_blocks(self.q, self.eb)[0]

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, push=None) -> torch.Tensor:
        from .._ext import ext
        t = x.shape[0]
        if out is None and push is None:
            out = torch.empty(t, self.N, dtype=torch.bfloat16, device=x.device)
        if t == 0:
            return out if push is None else push.push_args(0)[0]
        xq = torch.empty(t, self.K, dtype=torch.uint8, device=x.device)
        xs = torch.empty(t, self.K // TILE, dtype=torch.int32, device=x.device)
        ext().rmsnorm_quant(x.contiguous(), None, 0.0, 0.0, xq, xs, 0)
        return self.forward_quantized(xq, xs, out, push)

    def forward_quantized(self, xq: torch.Tensor, xs: torch.Tensor, out: torch.Tensor | None = None,
                          push=None) -> torch.Tensor:
        """y = dequant(xq, xs) W^T for activations already quantized (E4M3 [T, K] + UE8M0 words [T, K / 128]).
        push: a push-mode TPComm (see `DenseLinear`)."""
        t = xq.shape[0]
        pk = None
        if push is not None:
            out, *pk = push.push_args(t)
        if out is None:
            out = torch.empty(t, self.N, dtype=torch.bfloat16, device=xq.device)
        if t == 0:
            return out
        _splitk_gemm(self, xq, xs, out, t, self.K // TILE, 0, pk)
        return out


def act_quant(gate_up: torch.Tensor, gelu: bool = True, fmt: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """act(gate) * up over gate_up [T, 2F] (gate first), quantized in the same pass: fmt 0 -> (E4M3 [T, F], UE8M0
    words [T, F / 128]); fmt 1 -> (E2M1 pairs [T, F / 2], E4M3 scale bytes as words [T, F / 64]).  Equals quantizing
    the bf16 `act_mul` output bit for bit."""
    t, f = gate_up.shape[0], gate_up.shape[1] // 2
    if not gate_up.is_cuda:
        return act_quant_ref(gate_up, gelu, fmt)
    from .._ext import ext
    q = torch.empty(t, f if fmt == 0 else f // 2, dtype=torch.uint8, device=gate_up.device)
    sc = torch.empty(t, f // (128 if fmt == 0 else 64), dtype=torch.int32, device=gate_up.device)
    ext().act_quant(gate_up.contiguous(), gelu, q, sc, fmt)
    return q, sc


def act_quant_ref(gate_up: torch.Tensor, gelu: bool = True, fmt: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    from . import basic as B
    a = B.act_mul(gate_up.cpu(), gelu)
    return MG.quant_rows(a) if fmt == 0 else MG.quant_nvfp4_rows(a)


class Fp8Mlp:
    """Block-scaled FP8 gated MLP: gate_up GEMM -> fused act * up + per-128 quant -> down GEMM on the quantized
    activations (no bf16 intermediate round trip; the FP8 Gemma MLP glue of
    `attention/gemma-fused-glue/gelu_quant.py:1-30`)."""

    def __init__(self, w_gu: torch.Tensor, w_down: torch.Tensor, gelu: bool = True):
        self.gu, self.down, self.gelu = Fp8Linear(w_gu), Fp8Linear(w_down), gelu

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        h = self.gu(x)
        q, s = act_quant(h, self.gelu, 0)
        return self.down.forward_quantized(q, s)

    def reference(self, x: torch.Tensor) -> torch.Tensor:
        """fp32 oracle over the dequantized weights with the same activation quantization points."""
        from . import basic as B
        xq, xs = MG.quant_rows(x.float())
        h = (MG.dequant_rows(xq, xs) @ self.gu.dequant().float().t()).to(torch.bfloat16)
        a = B.act_mul(h.cpu(), self.gelu).float()
        aq, as_ = MG.quant_rows(a)
        return MG.dequant_rows(aq, as_) @ self.down.dequant().float().cpu().t()


class ShardedLMHead:
    """Vocabulary-parallel LM head: rank r holds rows [r V / n, (r + 1) V / n) (FP8 block-scaled or bf16) and returns
    its local (max logit, argmax) per token; `parallel.dist.argmax_merge` picks the global winner (ties: lower id),
    so the full logits never leave the GPU (the DP-LM-head shards of `moe-gemm/fp8-lm-head/pro_fp8_lm_head.py:59`)."""

    def __init__(self, w: torch.Tensor, rank: int, world: int, fp8: bool = True):
        V = w.shape[0]
        per = -(-V // world)
        self.v0 = rank * per
        shard = w[self.v0:min(V, self.v0 + per)]
        pad = (-shard.shape[0]) % 256
        if pad:
            shard = torch.cat([shard, torch.zeros(pad, w.shape[1], dtype=w.dtype, device=w.device)])
        self.rows = min(V, self.v0 + per) - self.v0
        self.lin = Fp8Linear(shard) if fp8 else DenseLinear(shard)

    def local_argmax(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        logits = self.lin(x)[:, :self.rows].float()
        val, idx = logits.max(-1)
        return val, idx + self.v0


class Linear:
    """A projection on this framework's GEMMs with any output width: W [N, K] (bf16 master) becomes an FP8 block-scaled
    (`fp8`) or bf16 (`bf16`) weight-streaming GEMM with the rows zero-padded to the kernel's 128-row tile; the result
    is the [T, N] view of the padded output.  `fuse` stacks several weights that read the same input into one launch
    (`split` returns the per-weight column views)."""

    def __init__(self, w: torch.Tensor, kind: str = "fp8"):
        N, K = w.shape
        self.N, self.K, self.kind = N, K, kind
        pad = (-N) % (256 if N > 128 else 128)
        wp = torch.cat([w, torch.zeros(pad, K, dtype=w.dtype, device=w.device)]) if pad else w
        self.lin = Fp8Linear(wp) if kind == "fp8" else DenseLinear(wp.to(torch.bfloat16))
        if kind == "fp8":
            self.lin.q = self.lin.eb = None          # the packed copy is the only one the GEMM reads
        self.Np = wp.shape[0]

    @classmethod
    def fuse(cls, ws: list, kind: str = "fp8") -> "Linear":
        lin = cls(torch.cat(ws), kind)
        lin.widths = [w.shape[0] for w in ws]
        return lin

    def __call__(self, x: torch.Tensor, out_f32: bool = False, push=None) -> torch.Tensor:
        """push: a push-mode `parallel.symm.TPComm` (row-parallel projection whose all-reduce follows; the output
        width must be the kernel's, no padding)."""
        if out_f32:
            assert self.kind == "bf16", "fp32 output is the bf16 GEMM's mode"
            y = self.lin(x, out_f32=True)
        elif push is not None:
            assert self.Np == self.N, "push: unpadded output width"
            y = self.lin(x, push=push)
        else:
            y = self.lin(x)
        return y[:, :self.N] if self.Np != self.N else y

    def partials(self, x: torch.Tensor) -> tuple[torch.Tensor, int]:
        """bf16 GEMM, fp32 split-K partials ([ks * t, N], ks) of x W^T, unpadded widths only (`DenseLinear.partials`)."""
        assert self.kind == "bf16" and self.Np == self.N, "partials: bf16 GEMM of an unpadded width"
        return self.lin.partials(x)

    def split(self, y: torch.Tensor) -> list:
        out, c = [], 0
        for w in self.widths:
            out.append(y[:, c:c + w])
            c += w
        return out


class HeadBatchedLinear:
    """Per-head projections y[t, h] = x[t, h] W[h]^T (W bf16 [H, N, K]) as ONE grouped bf16 GEMM launch: head h is
    "expert" h and every token is routed to every head, so the weights stream once at full tensor-core width (the
    MLA absorption products q_nope W_UK and o_lat W_UV).  Input rows are read in place: head h of token t is row
    t * row_stride + h of x viewed as [rows, K] (row_stride = H for a contiguous [T, H, K] input, larger when the
    heads sit inside a wider projection output).  Output: contiguous [T, H, N] bf16."""

    def __init__(self, w: torch.Tensor):
        H, N, K = w.shape
        assert N % TILE == 0 and K % 64 == 0 and H <= 1023
        self.H, self.N, self.K = H, N, K
        self.g = 2 if N % 256 == 0 else 1
        self.wpack = torch.cat([pack_bf16(w[h].to(torch.bfloat16), self.g) for h in range(H)])
        dev = w.device
        self.num_ctas = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 1
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._rows: dict = {}

    def _index(self, t: int, dev):
        """off [H + 1] = h t; pairs[h t + j] = j H + h (output row of token j, head h)."""
        if t not in self._rows:
            def make():
                h = torch.arange(self.H, dtype=torch.int32, device=dev)
                j = torch.arange(t, dtype=torch.int32, device=dev)
                return ((torch.arange(self.H + 1, dtype=torch.int32, device=dev) * t).contiguous(),
                        (j[None, :] * self.H + h[:, None]).reshape(-1).contiguous())
            self._rows[t] = MG.static_index_tensors(make)
        return self._rows[t]

    def __call__(self, x: torch.Tensor, t: int, row_stride: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """x: any tensor whose memory holds token t's head h at element (t * row_stride + h) * K (row_stride 0: H).
        out: optional [t H, >= N] bf16 view with unit column stride (e.g. the first N columns of a wider per-head
        row); default a new contiguous [t, H, N]."""
        rs = row_stride or self.H
        if out is None:
            out = torch.empty(t, self.H, self.N, dtype=torch.bfloat16, device=x.device)
        if t == 0:
            return out
        rows = x.reshape(-1).view(torch.uint8).view(-1, self.K * 2)
        off, pairs, static = self._index(t, x.device)
        MG.gemm(self.wpack, rows, rows, off, pairs, out.view(t * self.H, -1) if out.dim() == 3 else out, self.status,
                n_tiles=self.N // (TILE * self.g), kc=self.K // 64, g=self.g, nt=MG.pick_nt(t), mode=0, src_div=1,
                num_ctas=self.num_ctas, kind=2, src_group=self.H if rs != self.H else 0,
                src_group_stride=rs if rs != self.H else 0, static_index=static)
        return out
