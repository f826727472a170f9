"""Expert-parallel MoE over NVLink peer memory: dispatch by peer stores, grouped block-scaled expert GEMMs on the
local experts, expert outputs stored by the GEMM epilogue straight into the owning rank's combine buffer, and a
slot-ordered weighted combine on the owner (csrc/ep.cu, csrc/moe_gemm.cu).

Every rank holds `E_total / world` routed experts plus a replica of the shared expert (run on the rank's own tokens
as one more bucket of the same GEMM launches -- the reference's TP1-shared-under-DP arrangement,
`upstream-fixes/hooks/glm_tp1_shared_hooks.py`).  One symmetric allocation per group (torch symmetric-memory
rendezvous, mapped by every peer) holds, in this order:

    recv_x    [world * T_max, row_bytes]     quantized token rows, slot (src, t)
    recv_s    [world * T_max, scale_bytes]   their block scales
    recv_ids  [world * T_max, topk] int32    routing ids (-1: empty slot)
    comb      [T_max * topk + T_max, H] bf16 expert outputs of this rank's tokens (row t * topk + k), then the
                                             shared expert's rows
    flags     [world] int32                  barrier epochs

Per layer: quantize -> dispatch -> barrier -> align -> GEMM gate/up (+SwiGLU, requant) -> GEMM down (peer-store
epilogue) -> barrier -> combine.  A rank with no tokens runs the same launches (idle ranks join both barriers,
`moe-gemm/dp-moe-symmetric-memory/numinous_dp_moe.py:539-545`).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import ext
from ..ops import moe_gemm as MG


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class EPLayout:
    """Byte layout of the symmetric buffer (host-side arithmetic, testable without a GPU)."""

    def __init__(self, world: int, T_max: int, topk: int, H: int, fmt: str):
        self.world, self.T_max, self.topk, self.H = world, T_max, topk, H
        self.row_bytes = H if fmt == "fp8" else H // 2
        self.scale_words = H // 128 if fmt == "fp8" else H // 64
        rows = world * T_max
        self.off_x = 0
        self.off_s = _align(rows * self.row_bytes)
        self.off_ids = self.off_s + _align(rows * self.scale_words * 4)
        self.off_comb = self.off_ids + _align(rows * topk * 4)
        self.comb_rows = T_max * topk + T_max
        self.off_flags = self.off_comb + _align(self.comb_rows * H * 2)
        self.nbytes = self.off_flags + _align(world * 4)
        self.pairs_total = rows * topk

    def owner(self, expert: int, E_loc: int) -> int:
        return expert // E_loc

    def pair(self, src: int, t: int, k: int) -> int:
        """Pair id of slot k of token t of rank src (the GEMM row space of every rank)."""
        return (src * self.T_max + t) * self.topk + k

    def comb_row(self, pair: int) -> tuple[int, int]:
        """(rank, row) the expert output of `pair` is stored at."""
        d = self.T_max * self.topk
        return pair // d, pair % d


class EPComm:
    """The symmetric buffer, barrier epoch and scratch of the exchange: one per (group, T_max, shape), shared by every
    MoE layer of a model (layers run one after another, so one buffer serves them all and the epoch keeps counting)."""

    def __init__(self, rank: int, world: int, T_max: int, topk: int, H: int, F: int, fmt: str, E_loc: int,
                 has_shared: bool, device, group=None):
        import torch.distributed._symmetric_memory as symm
        self.rank, self.world, self.T_max, self.topk, self.E_loc = rank, world, T_max, topk, E_loc
        kind = 0 if fmt == "fp8" else 1
        L = self.layout = EPLayout(world, T_max, topk, H, fmt)
        self.buf = symm.empty(L.nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.group = grp
        self.handle = symm.rendezvous(self.buf, grp)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=device)
        rows = world * T_max
        self.recv_x = self.buf[L.off_x:L.off_x + rows * L.row_bytes].view(rows, L.row_bytes)
        self.recv_s = self.buf[L.off_s:L.off_s + rows * L.scale_words * 4].view(torch.int32).view(rows, L.scale_words)
        self.recv_ids = self.buf[L.off_ids:L.off_ids + rows * topk * 4].view(torch.int32)
        self.comb = self.buf[L.off_comb:L.off_comb + L.comb_rows * H * 2].view(torch.bfloat16).view(L.comb_rows, H)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.xq = torch.zeros(T_max, L.row_bytes, dtype=torch.uint8, device=device)
        self.xs = torch.zeros(T_max, L.scale_words, dtype=torch.int32, device=device)
        nb = E_loc + (1 if has_shared else 0)
        self.off = torch.zeros(nb + 1, dtype=torch.int32, device=device)
        self.pairs = torch.zeros(L.pairs_total + T_max, dtype=torch.int32, device=device)
        hb = F if kind == 0 else F // 2
        hw = F // 128 if kind == 0 else F // 64
        self.h = torch.zeros(L.pairs_total + T_max, hb, dtype=torch.uint8, device=device)
        self.hs = torch.zeros(L.pairs_total + T_max, hw, dtype=torch.int32, device=device)
        self.nt = MG.tactic_nt(world * T_max, fmt) or MG.pick_nt(max(1, -(-2 * L.pairs_total // (world * E_loc))))
        torch.cuda.synchronize(device)
        dist.barrier(group=grp)


class EPMoE:
    def __init__(self, rank: int, world: int, E_total: int, T_max: int, topk: int, w_gate: torch.Tensor = None,
                 w_up: torch.Tensor = None, w_down: torch.Tensor = None, shared: tuple | None = None,
                 fmt: str = "fp8", group=None, experts: MG.BlockScaledExperts | None = None,
                 comm: EPComm | None = None):
        """w_gate / w_up [E_loc, F, H], w_down [E_loc, H, F]: this rank's experts (global ids rank * E_loc ..);
        or `experts`: an already packed BlockScaledExperts of this rank's E_loc experts.  `comm`: a shared EPComm
        (the layers of one model share it); None allocates one for this layer (a collective)."""
        self.rank, self.world, self.T_max, self.topk = rank, world, T_max, topk
        self.E_loc = E_total // world
        if experts is None:
            assert w_gate.shape[0] == self.E_loc, "pass this rank's slice of the experts"
            experts = MG.BlockScaledExperts(w_gate, w_up, w_down, shared=shared, fmt=fmt)
        self.ex = experts
        self.fmt, self.kind, self.H, self.F = experts.fmt, self.ex.kind, self.ex.H, self.ex.F
        if comm is None:
            comm = EPComm(rank, world, T_max, topk, self.H, self.F, self.fmt, self.E_loc, experts.has_shared,
                          experts.w1.device, group)
        assert (comm.T_max, comm.topk, comm.world, comm.E_loc) == (T_max, topk, world, self.E_loc)
        self.comm = comm
        self.use_nccl = False             # True: `forward` runs the NCCL baseline exchange (`forward_nccl`)
        for name in ("layout", "buf", "handle", "peers", "recv_x", "recv_s", "recv_ids", "comb", "epoch", "status",
                     "xq", "xs", "off", "pairs", "h", "hs", "nt", "group"):
            setattr(self, name, getattr(comm, name))

    def barrier(self) -> None:
        ext().ep_barrier(self.peers, self.layout.off_flags, self.rank, self.world, self.epoch, self.status)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, xq8: tuple | None = None) -> torch.Tensor:
        """x bf16 [T, H] normalized, ids int32 [T, topk] global expert ids, w fp32 [T, topk] -> bf16 [T, H].
        xq8: (E4M3 [T, H], scales [T, H / 128]) when the norm that produced x already quantized it (FP8 experts)."""
        if self.use_nccl:
            return self.forward_nccl(x, ids, w, xq8)
        L, ex = self.layout, self.ex
        T, k = ids.shape
        if T > self.T_max:
            raise ValueError(f"{T} tokens > T_max {self.T_max}")
        xq, xs = self.xq[:T], self.xs[:T]
        if xq8 is not None and self.kind == 0 and T:
            xq, xs = xq8
        elif T:
            ext().rmsnorm_quant(x.contiguous(), None, 0.0, 0.0, xq, xs, self.kind)
        ext().ep_dispatch(self.peers, xq, xs, ids.contiguous(), L.off_x, L.off_s, L.off_ids, self.T_max, self.rank,
                          self.world, self.E_loc)
        self.barrier()
        extra = T if ex.has_shared else 0
        ext().moe_align(self.recv_ids, self.rank * self.E_loc, self.E_loc, extra, self.off, self.pairs)
        P = L.pairs_total
        vals = 128 if self.kind == 0 else 256
        MG.gemm(ex.w1, self.recv_x, self.recv_s, self.off, self.pairs, self.h, self.status,
                n_tiles=self.F // 128, kc=self.H // vals, g=2, nt=self.nt, mode=1, src_div=k,
                src_limit=P, src_shared_base=self.rank * self.T_max, out_scale=self.hs, num_ctas=ex.num_ctas,
                kind=self.kind, expert_mul=ex.mul1)
        # off / pairs were complete before the gate/up GEMM passed its dependency wait: this launch may build its work
        # list and stream weights while that GEMM finishes
        MG.gemm(ex.w2, self.h, self.hs, self.off, self.pairs, self.comb, self.status,
                n_tiles=self.H // (128 * ex.g2), kc=self.F // vals, g=ex.g2, nt=self.nt, mode=0, src_div=1,
                num_ctas=ex.num_ctas, kind=self.kind, expert_mul=ex.mul2, out_peers=self.peers,
                out_offset=L.off_comb, out_div=self.T_max * k, out_rank=self.rank,
                out_shared_base=self.T_max * k, pairs_total=P, static_index=True)
        self.barrier()
        y = torch.empty(T, self.H, dtype=torch.bfloat16, device=x.device)
        ext().moe_combine(self.comb, T, k, self.T_max * k if ex.has_shared else -1, w.float().contiguous(), y)
        return y

    def forward_nccl(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor,
                     xq8: tuple | None = None) -> torch.Tensor:
        """The same exchange over NCCL collectives instead of peer memory -- the baseline of the fused path and its
        correctness reference: quantized rows, scales and ids all-gathered (padded to T_max), the same grouped GEMMs
        on local buffers, every rank's expert rows returned to their token's rank by one all-to-all, each row taken
        from its expert's owner, the same slot-order combine.  Every value is computed by the same kernels at the
        same rounding points, so the output equals `forward`'s bit for bit."""
        L, ex, grp = self.layout, self.ex, self.group
        T, k = ids.shape
        if T > self.T_max:
            raise ValueError(f"{T} tokens > T_max {self.T_max}")
        dev, Tm, W = x.device, self.T_max, self.world
        xq = torch.zeros(Tm, L.row_bytes, dtype=torch.uint8, device=dev)
        xs = torch.zeros(Tm, L.scale_words, dtype=torch.int32, device=dev)
        if T:
            if xq8 is not None and self.kind == 0:
                xq[:T], xs[:T] = xq8
            else:
                ext().rmsnorm_quant(x.contiguous(), None, 0.0, 0.0, xq[:T], xs[:T], self.kind)
        idp = torch.full((Tm, k), -1, dtype=torch.int32, device=dev)
        idp[:T] = ids
        rx = torch.empty(W * Tm, L.row_bytes, dtype=torch.uint8, device=dev)
        rs = torch.empty(W * Tm, L.scale_words, dtype=torch.int32, device=dev)
        ri = torch.empty(W * Tm * k, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(rx, xq, group=grp)
        dist.all_gather_into_tensor(rs, xs, group=grp)
        dist.all_gather_into_tensor(ri, idp.view(-1), group=grp)
        extra = T if ex.has_shared else 0
        ext().moe_align(ri, self.rank * self.E_loc, self.E_loc, extra, self.off, self.pairs)
        P = L.pairs_total
        vals = 128 if self.kind == 0 else 256
        MG.gemm(ex.w1, rx, rs, self.off, self.pairs, self.h, self.status,
                n_tiles=self.F // 128, kc=self.H // vals, g=2, nt=self.nt, mode=1, src_div=k,
                src_limit=P, src_shared_base=self.rank * Tm, out_scale=self.hs, num_ctas=ex.num_ctas,
                kind=self.kind, expert_mul=ex.mul1)
        rows = torch.empty(P + Tm, self.H, dtype=torch.bfloat16, device=dev)   # row = pair id; shared: P + t
        MG.gemm(ex.w2, self.h, self.hs, self.off, self.pairs, rows, self.status,
                n_tiles=self.H // (128 * ex.g2), kc=self.F // vals, g=ex.g2, nt=self.nt, mode=0, src_div=1,
                num_ctas=ex.num_ctas, kind=self.kind, expert_mul=ex.mul2)
        back = torch.empty(P, self.H, dtype=torch.bfloat16, device=dev)        # block q: my pairs as rank q saw them
        dist.all_to_all_single(back, rows[:P], group=grp)
        comb = torch.zeros(L.comb_rows, self.H, dtype=torch.bfloat16, device=dev)
        if T:
            slot = torch.arange(T * k, device=dev)
            owner = (ids.reshape(-1).long() // self.E_loc).clamp(0, W - 1)
            comb[:T * k] = back[owner * (Tm * k) + slot]
            if ex.has_shared:
                comb[Tm * k:Tm * k + T] = rows[P:P + T]
        y = torch.empty(T, self.H, dtype=torch.bfloat16, device=dev)
        ext().moe_combine(comb, T, k, Tm * k if ex.has_shared else -1, w.float().contiguous(), y)
        return y

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError(f"expert-parallel exchange: status {int(self.status.item())}")


class EPMoERef:
    """Expert parallelism by plain collectives (any backend; gloo on the CPU): token rows, ids and weights of every
    rank are all-gathered (padded to T_max), each rank applies its E / world routed experts to every pair routed to
    them and its shared-expert replica to its own tokens, and a sum all-reduce hands every rank its rows.  Same
    interface and lockstep contract as `EPMoE` (every rank calls forward for every MoE layer, idle ranks with T = 0);
    the host-side oracle of the expert-parallel serving loop."""

    def __init__(self, rank: int, world: int, E_total: int, T_max: int, topk: int, w_gu: torch.Tensor,
                 w_down: torch.Tensor, shared: tuple | None = None, group=None):
        self.rank, self.world, self.T_max, self.topk = rank, world, T_max, topk
        self.E_loc = E_total // world
        assert w_gu.shape[0] == self.E_loc, "pass this rank's slice of the experts"
        self.w_gu, self.w_down, self.shared, self.group = w_gu, w_down, shared, group
        self.H = w_down.shape[1]

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, xq8: tuple | None = None) -> torch.Tensor:
        from ..ops import moe as MOE
        T, k = ids.shape
        if T > self.T_max:
            raise ValueError(f"{T} tokens > T_max {self.T_max}")
        dev = x.device
        xp = torch.zeros(self.T_max, self.H, dtype=x.dtype, device=dev)
        ip = torch.full((self.T_max, k), -1, dtype=torch.int32, device=dev)
        wp = torch.zeros(self.T_max, k, dtype=torch.float32, device=dev)
        xp[:T], ip[:T], wp[:T] = x, ids, w.float()
        xs = [torch.empty_like(xp) for _ in range(self.world)]
        is_ = [torch.empty_like(ip) for _ in range(self.world)]
        ws = [torch.empty_like(wp) for _ in range(self.world)]
        dist.all_gather(xs, xp, group=self.group)
        dist.all_gather(is_, ip, group=self.group)
        dist.all_gather(ws, wp, group=self.group)
        X, I, W = torch.cat(xs), torch.cat(is_), torch.cat(ws)
        out = MOE.experts_ref(X, I, W, self.w_gu, self.w_down, self.rank * self.E_loc)
        if self.shared is not None and T:
            out[self.rank * self.T_max:self.rank * self.T_max + T] += MOE.swiglu(x, *self.shared).float()
        dist.all_reduce(out, group=self.group)
        return out[self.rank * self.T_max:self.rank * self.T_max + T].to(torch.bfloat16)

    def check(self) -> None:
        pass
