"""Model runner for the GQA family: turns scheduled segments into device step tensors, runs prefill (eager) and
decode / speculative steps (CUDA graphs per batch bucket), and samples greedily.

Step inputs travel as ONE pinned int32 staging buffer copied host->device per step (ids, positions, pool slots per
layer kind, per-group kv lengths and page-table rows); the page tables are synced the same way.  Results come back as
one device->host copy of the sampled ids.  This is the engine's whole per-step host traffic, which is what bench.py's
end-to-end number accounts for.

Attention runs every mode (prefill chunks, decode, verify, draft extend) through the same split-K kernel: a segment
of L tokens is cut into groups of n_q consecutive tokens (n_q * G <= 16 query rows per kv head); a group's last
rows may be padding (slot -1, output discarded), which is safe because a query only sees keys at or before its own
position.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch

from ..config import EngineConfig, GQAConfig
from ..kv.allocator import RequestPages
from ..models.gqa import GQAKVCache, GQAModel, StepTensors
from ..ops import attention as A
from ..ops import basic as B
from ..ops import kvcache as K
from .scheduler import SamplingParams, Batch, Request, Segment

KINDS = ("global", "swa", "draft")


@dataclass
class Packed:
    ids: list
    pos: list
    slot: dict
    kv_len: list
    req_idx: list
    n_q: int
    logit_rows: list            # row index per segment that wants logits
    seg_rows: list              # (segment, first row) for each segment


class StagingBuffers:
    """One device int32 buffer holding every per-step input, plus its pinned host twin."""

    def __init__(self, max_tokens: int, max_groups: int, kinds: tuple, device):
        self.kinds = kinds
        self.T, self.G = max_tokens, max_groups
        n = max_tokens * (2 + len(kinds)) + 2 * max_groups
        pin = torch.device(device).type == "cuda"
        self.host = torch.zeros(n, dtype=torch.int32, pin_memory=pin)
        self.dev = torch.zeros(n, dtype=torch.int32, device=device)

    def views(self, buf: torch.Tensor, t: int, g: int):
        T, G = self.T, self.G
        ids, pos = buf[:t], buf[T:T + t]
        slots = {k: buf[(2 + i) * T:(2 + i) * T + t] for i, k in enumerate(self.kinds)}
        base = (2 + len(self.kinds)) * T
        return ids, pos, slots, buf[base:base + g], buf[base + G:base + G + g]

    def fill(self, p: Packed) -> None:
        t, g = len(p.ids), len(p.kv_len)
        ids, pos, slots, kvl, rix = self.views(self.host, t, g)
        ids.copy_(torch.tensor(p.ids, dtype=torch.int32))
        pos.copy_(torch.tensor(p.pos, dtype=torch.int32))
        for k in self.kinds:
            slots[k].copy_(torch.tensor(p.slot.get(k, [-1] * t), dtype=torch.int32))
        kvl.copy_(torch.tensor(p.kv_len, dtype=torch.int32))
        rix.copy_(torch.tensor(p.req_idx, dtype=torch.int32))

    def upload(self) -> None:
        self.dev.copy_(self.host, non_blocking=True)

    def step_tensors(self, t: int, g: int, n_q: int, splits: dict) -> StepTensors:
        ids, pos, slots, kvl, rix = self.views(self.dev, t, g)
        return StepTensors(ids, pos, slots, kvl, rix, n_q, splits)

    def h2d_bytes(self) -> int:
        return self.host.numel() * 4


class GQARunner:
    def __init__(self, cfg: GQAConfig, ecfg: EngineConfig, device, max_seq: int, tp_rank: int = 0, tp: int = 1,
                 all_reduce: Optional[Callable] = None, argmax_merge: Optional[Callable] = None,
                 global_pages: Optional[int] = None):
        if ecfg.kv_dtype == "kvmix":
            raise ValueError("kv_dtype 'kvmix' (FP8 + NVFP4 latent rows in one page space) is an MLA-family pool")
        self.cfg, self.ecfg, self.device = cfg, ecfg, torch.device(device)
        self.tp, self.tp_rank = tp, tp_rank
        self.max_seq = max_seq
        self.argmax_merge = argmax_merge
        ck = None
        if ecfg.checkpoint:                          # this rank's tensor-parallel shards of a HuggingFace checkpoint
            from ..models.loader import open_checkpoint, shard_gqa
            ck = open_checkpoint(ecfg.checkpoint)
        self.model = GQAModel(cfg, device, tp_rank, tp, ecfg.seed, all_reduce,
                              weights=shard_gqa(ck, cfg, tp_rank, tp, device) if ck else None)
        self.spec = ecfg.spec
        self.n_draft = ecfg.draft_tokens if ecfg.spec else 0
        self.draft = GQAModel(cfg, device, tp_rank, tp, ecfg.seed, all_reduce, draft=True,
                              weights=shard_gqa(ck, cfg, tp_rank, tp, device, draft=True) if ck else None) \
            if self.spec else None
        self.tp_comm = None
        self.qar = None
        if tp > 1 and ecfg.tp_qar and self.device.type == "cuda":
            # FP8 two-shot all-reduce (csrc/qar.cu) as the model's all-reduce; the norms run as their own kernels
            from ..parallel.qar import QuantAllReduce
            # a packed prefill batch pads every segment to a multiple of its query group (<= 16 tokens)
            rows = max(ecfg.chunked_prefill, 4 * max(ecfg.graph_sizes() + [ecfg.max_running])) + \
                16 * (ecfg.max_running + 1)
            self.qar = QuantAllReduce(tp_rank, tp, rows, cfg.hidden, self.device)
            for m in (self.model, self.draft):
                if m is not None:
                    m.all_reduce = self.qar
        elif tp > 1 and ecfg.fused_comm and self.device.type == "cuda":
            from ..parallel.symm import TPComm
            rows = max(ecfg.chunked_prefill, 4 * max(ecfg.graph_sizes() + [ecfg.max_running]))
            push = (ecfg.tp_push and not ecfg.tp_nvls and self.model.can_push()
                    and (self.draft is None or self.draft.can_push()))
            self.tp_comm = TPComm(tp_rank, tp, rows, cfg.hidden, self.device, push=push, nvls=ecfg.tp_nvls)
            self.model.tp_comm = self.tp_comm
            if self.draft is not None:
                self.draft.tp_comm = self.tp_comm
        G = cfg.num_q_heads // cfg.num_kv_heads
        self.n_q_prefill = max(1, 16 // G)
        self.max_running = ecfg.max_running
        w = cfg.sliding_window
        per_req_swa = (w + self.ecfg.chunked_prefill) // 64 + 3
        swa_pages = self.max_running * (w // 64 + 4) + per_req_swa + 2
        if global_pages is None:
            # global-layer pages (sliding-window pools are sized by the window): the requests' need, bounded by
            # max_total_tokens / mem_fraction of the memory free at boot
            from .mla_runner import pool_pages
            fmt = K.FMT_IDS[ecfg.kv_dtype]
            n_glob = sum(1 for i in range(cfg.num_layers) if cfg.is_global(i))
            page_bytes = n_glob * (cfg.num_kv_heads_global // tp) * 2 * K.part_bytes(fmt, cfg.head_dim_global)
            global_pages = pool_pages(ecfg, self.max_running * ((max_seq + 64 + 63) // 64) + 2, page_bytes, device)
        self.pool_tokens = 64 * (global_pages - 2)
        self.kv = GQAKVCache(cfg, tp, device, ecfg.kv_dtype, self.max_running + 1, max_seq + 64, global_pages,
                             swa_pages, draft_pages=swa_pages if self.spec else 0)
        self.dummy_row = self.max_running
        self.pages: dict[int, dict[str, RequestPages]] = {}
        max_tok = max(ecfg.chunked_prefill + 16 * self.n_q_prefill, self.max_running * (self.n_draft + 1))
        self.max_tok = max_tok
        self.max_groups = max_tok
        self.stage = StagingBuffers(max_tok, self.max_groups, KINDS, device)
        self.kv.reserve_workspace(self.max_running, self._max_splits())
        self.graphs: dict = {}
        self.graph_pool = None
        self.out_ids = torch.zeros(max_tok, dtype=torch.int32, device=device)
        pin = self.device.type == "cuda"
        self.out_host = torch.zeros(max_tok, dtype=torch.int32, pin_memory=pin)
        if self.spec:
            self._init_spec()

    # ------------------------------------------------------------------------------------------ memory
    def _max_splits(self) -> int:
        best = 1
        for kind, hk in (("global", self.cfg.num_kv_heads_global // self.tp), ("swa", self.cfg.num_kv_heads // self.tp)):
            for b in range(1, self.max_running + 1):
                best = max(best, A.split_policy(b * hk, self.max_seq, self.cfg.sliding_window if kind == "swa" else 0)[0])
        return best

    def can_admit(self, r: Request) -> bool:
        need = (r.prompt_len + r.params.max_new_tokens + self.n_draft + 64) // 64 + 1
        return self.kv.alloc["global"].free >= need + self._reserved_growth()

    def _reserved_growth(self) -> int:
        tot = 0
        for rid, pg in self.pages.items():
            tot += max(0, pg["_max_pages"] - len(pg["global"].pages))
        return tot

    def attach(self, r: Request) -> None:
        w = self.cfg.sliding_window
        pg = {"global": RequestPages(self.kv.alloc["global"], self.kv.tables["global"], r.slot),
              "swa": RequestPages(self.kv.alloc["swa"], self.kv.tables["swa"], r.slot, window=w)}
        if self.spec:
            pg["draft"] = RequestPages(self.kv.alloc["draft"], self.kv.tables["draft"], r.slot, window=w)
        pg["_max_pages"] = (r.prompt_len + r.params.max_new_tokens + self.n_draft + 64) // 64 + 1
        self.pages[r.rid] = pg

    def detach(self, r: Request) -> None:
        pg = self.pages.pop(r.rid, None)
        if pg:
            for k in KINDS:
                if k in pg:
                    pg[k].free()

    # ------------------------------------------------------------------------------------------ packing
    def _pack(self, segs: list, n_q: int, kinds: tuple, pad_groups_to: int = 0, draft_offset: int = 0) -> Packed:
        ids, pos, kvl, rix, logit_rows, seg_rows = [], [], [], [], [], []
        slot = {k: [] for k in kinds}
        for s in segs:
            L = len(s.tokens)
            ngroups = (L + n_q - 1) // n_q
            pg = self.pages[s.req.rid]
            for k in kinds:
                pg[k].ensure(s.start + L + draft_offset)
            seg_rows.append((s, len(ids)))
            for gi in range(ngroups):
                for t in range(n_q):
                    j = gi * n_q + t
                    p = s.start + j
                    if j < L:
                        ids.append(int(s.tokens[j]))
                        pos.append(p)
                        for k in kinds:
                            slot[k].append(pg[k].slot_of(p))
                    else:
                        ids.append(0)
                        pos.append(p)
                        for k in kinds:
                            slot[k].append(-1)
                kvl.append(s.start + (gi + 1) * n_q)
                rix.append(s.req.slot)
            if s.logits:
                logit_rows.append(seg_rows[-1][1] + L - 1)
        while len(kvl) < pad_groups_to:
            for t in range(n_q):
                ids.append(0)
                pos.append(t)
                for k in kinds:
                    slot[k].append(-1)
            kvl.append(n_q)
            rix.append(self.dummy_row)
        p = Packed(ids, pos, slot, kvl, rix, n_q, logit_rows, seg_rows)
        if self.ecfg.bounds_check:
            from ..tooling.bounds import check_gqa_pack
            self.kv.sync_tables()
            check_gqa_pack(p, self.kv, self.max_running + 1)
        return p

    def _ext_segs(self, p: Packed) -> Optional[list]:
        """Prefill segments for the extend kernel: (first q row, real tokens, first position, page-table row)."""
        if not self.ecfg.extend_kernel:
            return None
        return [(r0, len(s.tokens), s.start, s.req.slot) for s, r0 in p.seg_rows]

    # ------------------------------------------------------------------------------------------ forward pieces
    def _target(self, st: StepTensors):
        return self.model.forward(st, self.kv)

    def _greedy(self, x_sel: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        logits = self.model.logits_local(x_sel, self.model.embed)
        if self.tp == 1:
            return B.argmax(logits, out=out[: x_sel.shape[0]])
        val = torch.empty(x_sel.shape[0], dtype=torch.float32, device=self.device)
        loc = B.argmax(logits, val=val)
        return self.argmax_merge(loc, val, self.model.vocab_local, out[: x_sel.shape[0]])

    # ------------------------------------------------------------------------------------------ prefill
    def prefill(self, batch: Batch) -> dict:
        for s in batch.segments:
            if s.req.rid not in self.pages:
                self.attach(s.req)
        kinds = ("global", "swa", "draft") if self.spec else ("global", "swa")
        p = self._pack(batch.segments, self.n_q_prefill, kinds)
        self.kv.sync_tables()
        self.stage.fill(p)
        self.stage.upload()
        st = self.stage.step_tensors(len(p.ids), len(p.kv_len), p.n_q,
                                     {"global": (1, 1 << 20), "swa": (1, 1 << 20), "draft": (1, 1 << 20)})
        st.ext_segs = self._ext_segs(p)
        x, resid = self._target(st)
        rows = torch.tensor(p.logit_rows, dtype=torch.long, device=self.device)
        res = {}
        if len(p.logit_rows):
            self._greedy(x[rows], self.out_ids)
            self.out_host[: len(p.logit_rows)].copy_(self.out_ids[: len(p.logit_rows)], non_blocking=True)
        if self.spec:
            self._draft_prefill(batch, p, resid, st)
            for s, r0 in p.seg_rows:
                if s.logits:   # target hidden of the last prompt position: the first draft step's input
                    self.hbuf[s.req.slot, 0].copy_(resid[r0 + len(s.tokens) - 1])
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        k = 0
        for s in batch.segments:
            if s.logits:
                res[s.req.rid] = int(self.out_host[k])
                s.req.draft_state["ld"] = s.start + len(s.tokens)   # draft KV exact below this position
                k += 1
        self._trim(batch.segments)
        return res

    # ------------------------------------------------------------------------------------------ split prefill
    # The prefill lane of the SM-partitioned prefill / decode lanes (engine/pdmux.py): one prefill chunk advances a
    # few decoder layers per engine iteration on its own stream while decode steps run on the other lane's stream
    # (`parallelism/in-node-pd-disaggregation/glm_pdmux_split_hooks.py:1-30`).  The lane has its own staging
    # buffers and output ids; the decode lane keeps `self.stage`.
    def split_begin(self, batch: Batch) -> dict:
        if self.spec or self.tp != 1:
            raise NotImplementedError("split prefill lanes: speculative decoding and tp > 1 are not supported")
        if not hasattr(self, "p_stage"):
            self.p_stage = StagingBuffers(self.max_tok, self.max_groups, KINDS, self.device)
            self.p_out = torch.zeros(self.max_tok, dtype=torch.int32, device=self.device)
            self.p_out_host = torch.zeros(self.max_tok, dtype=torch.int32, pin_memory=self.device.type == "cuda")
        for s in batch.segments:
            if s.req.rid not in self.pages:
                self.attach(s.req)
        p = self._pack(batch.segments, self.n_q_prefill, ("global", "swa"))
        self.kv.sync_tables()
        self.p_stage.fill(p)
        self.p_stage.upload()
        st = self.p_stage.step_tensors(len(p.ids), len(p.kv_len), p.n_q, {"global": (1, 1 << 20),
                                                                          "swa": (1, 1 << 20)})
        st.ext_segs = self._ext_segs(p)
        st.lane = 1
        return {"batch": batch, "p": p, "st": st, "x": None, "resid": None, "index": 0}

    def split_layers(self, sp: dict, count: int) -> bool:
        """Enqueue layers [index, index + count) of the split on the current stream; after the last layer also the
        logits / argmax of the rows that want a token.  Returns True when the split's device work is all enqueued.
        Its launches use the lane's own split-K scratch (`moe_gemm.LANE`): decode may run concurrently on another
        stream with a batch of the same size."""
        from ..ops import moe_gemm as MG
        MG.LANE[0] = 1
        try:
            return self._split_layers(sp, count)
        finally:
            MG.LANE[0] = 0

    def _split_layers(self, sp: dict, count: int) -> bool:
        n_layers = len(self.model.layers)
        lo = sp["index"]
        hi = min(lo + max(1, count), n_layers)
        sp["x"], sp["resid"] = self.model.forward_layers(sp["st"], self.kv, lo, hi, sp["x"], sp["resid"])
        sp["index"] = hi
        if hi < n_layers:
            return False
        p = sp["p"]
        if len(p.logit_rows):
            rows = torch.tensor(p.logit_rows, dtype=torch.long)     # pinned + async: the host never waits on the lane
            rows = rows.pin_memory().to(self.device, non_blocking=True) if self.device.type == "cuda" else rows
            self._greedy(sp["x"][rows], self.p_out)
            self.p_out_host[: len(p.logit_rows)].copy_(self.p_out[: len(p.logit_rows)], non_blocking=True)
        sp["x"] = sp["resid"] = None
        return True

    def split_finish(self, sp: dict) -> dict:
        """Host side of a finished split, after its stream's work completed: rid -> first generated token."""
        res, k = {}, 0
        for s in sp["batch"].segments:
            if s.logits:
                res[s.req.rid] = int(self.p_out_host[k])
                s.req.draft_state["ld"] = s.start + len(s.tokens)
                k += 1
        self._trim(sp["batch"].segments)
        return res

    @torch.no_grad()
    def score(self, tokens: list) -> torch.Tensor:
        """Teacher-forced full logits [T, V] (fp32, CPU) of one sequence through the paged pool (tp = 1): the
        accuracy gate's input.  Uses a scratch request row; nothing stays allocated."""
        if self.tp != 1:
            raise NotImplementedError("score() gathers logits on one rank")
        r = Request(rid=-1, prompt=list(tokens), params=SamplingParams(max_new_tokens=1))
        r.slot = next(i for i in range(self.max_running) if all(p["global"].slot != i for p in self.pages.values()))
        self.attach(r)
        try:
            kinds = ("global", "swa", "draft") if self.spec else ("global", "swa")
            p = self._pack([Segment(r, 0, list(tokens), True)], self.n_q_prefill, kinds)
            self.kv.sync_tables()
            self.stage.fill(p)
            self.stage.upload()
            st = self.stage.step_tensors(len(p.ids), len(p.kv_len), p.n_q,
                                         {"global": (1, 1 << 20), "swa": (1, 1 << 20), "draft": (1, 1 << 20)})
            st.ext_segs = self._ext_segs(p)
            x, _ = self._target(st)
            rows = torch.arange(len(tokens), device=self.device)
            return self.model.logits_local(x[rows], self.model.embed).float().cpu()
        finally:
            self.detach(r)

    def _trim(self, segs) -> None:
        for s in segs:
            pg = self.pages.get(s.req.rid)
            if pg is None:
                continue
            nxt = s.start + len(s.tokens)
            pg["swa"].trim(nxt)
            if "draft" in pg:
                pg["draft"].trim(nxt)

    # ------------------------------------------------------------------------------------------ decode
    def _bucket(self, n: int) -> int:
        for b in self.ecfg.graph_sizes():
            if b >= n:
                return b
        return n

    def decode(self, reqs: list) -> dict:
        """One greedy decode step (n_q = 1) for every running request."""
        segs = [Segment(r, r.kv_len, [r.pending], True) for r in reqs]
        bucket = self._bucket(len(segs))
        p = self._pack(segs, 1, ("global", "swa"), pad_groups_to=bucket)
        self.kv.sync_tables()
        self.stage.fill(p)
        self.stage.upload()
        fn = self._decode_fn(bucket)
        self._timed(fn)
        n = len(segs)
        self.out_host[:n].copy_(self.out_ids[:n], non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        res = {r.rid: [int(self.out_host[i])] for i, r in enumerate(reqs)}
        if self.spec:
            self._keep_draft_inputs(reqs)
        self._trim([Segment(r, r.kv_len, [0], False) for r in reqs])
        return res

    def draft_row(self, r) -> int:
        """Row of the stored target hiddens that a plain decode step of `r` fills: the next draft extend covers
        positions [ld, L] with inputs h_{ld-1} .. h_{L-1} in rows 0 .. L - ld."""
        return r.kv_len - r.draft_state.get("ld", r.kv_len) + 1

    def _keep_draft_inputs(self, reqs: list) -> None:
        """After a plain decode step on a speculative engine: store each request's new target hidden where the next
        draft extend reads it, or mark the request's draft stale when the extend window (4 positions) is full."""
        if not hasattr(self, "hbuf"):
            self._init_spec()
        h = self.cfg.hidden
        if all(r.draft_state.get("stale") for r in reqs):
            return
        dummy = self.hbuf.shape[0] - 1
        idx = []
        for r in reqs:
            row = self.draft_row(r)
            if 0 <= row <= 3 and not r.draft_state.get("stale"):
                idx.append(r.slot * 4 + row)
            else:
                r.draft_state["stale"] = True
                idx.append(dummy * 4)
        dev = torch.tensor(idx, dtype=torch.long).to(self.device, non_blocking=True)
        self.hbuf.view(-1, h).index_copy_(0, dev, self.dec_resid[:len(reqs)])

    def _timed(self, fn: Callable) -> None:
        """Run a step body; when `self.event_log` is a list, bracket it with CUDA events (device time of the step
        computation without host staging) and append the pair."""
        if getattr(self, "event_log", None) is not None and self.device.type == "cuda":
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            self.event_log.append((e0, e1))
        else:
            fn()

    def count_step_launches(self, bucket: int, kind: Optional[str] = None) -> int:
        """Kernel launches (of this package's extension) in one decode step body, run eagerly under the counter;
        kind "spec" | "decode" (default: the engine's configured mode)."""
        from .._ext import count_launches
        spec = self.spec if kind is None else kind == "spec"
        body = self._spec_body(bucket) if spec else self._decode_body(bucket)
        with count_launches() as c:
            body()
        return c.n

    def _splits(self, groups: int) -> dict:
        cfg = self.cfg
        return {"global": A.split_policy(groups * cfg.num_kv_heads_global // self.tp, self.max_seq),
                "swa": A.split_policy(groups * cfg.num_kv_heads // self.tp, self.max_seq, cfg.sliding_window),
                "draft": A.split_policy(groups * cfg.num_kv_heads // self.tp, self.max_seq, cfg.sliding_window)}

    def _decode_body(self, bucket: int) -> Callable:
        st = self.stage.step_tensors(bucket, bucket, 1, self._splits(bucket))

        def body():
            x, resid = self._target(st)
            self._greedy(x, self.out_ids)
            if self.spec:
                self.dec_resid[:bucket].copy_(resid[:bucket])
        return body

    def _decode_fn(self, bucket: int) -> Callable:
        key = ("decode", bucket)
        if key in self.graphs:
            return self.graphs[key]
        body = self._decode_body(bucket)
        if not (self.ecfg.cuda_graphs and self.device.type == "cuda"):
            self.graphs[key] = body
            return body
        fn = self._capture(body)
        self.graphs[key] = fn
        return fn

    def has_graph(self, n: int) -> bool:
        """The decode graph of n's batch bucket is captured."""
        return ("decode", self._bucket(n)) in self.graphs

    def warm_graphs(self, n: int) -> None:
        """Capture the decode (and speculative) graphs of n's batch bucket on padding-only inputs (no KV writes, the
        dummy request row), so that capture never lands inside a timed or policy-priced step."""
        bucket = self._bucket(n)
        self.stage.fill(self._pack([], 1, ("global", "swa"), pad_groups_to=bucket))
        self.stage.upload()
        self._decode_fn(bucket)
        if self.spec:
            if not hasattr(self, "hbuf"):
                self._init_spec()
            for st, nq, kinds in ((self.st_ext, 4, ("draft",)), (self.st_d2, 1, ("draft",)),
                                  (self.st_d3, 1, ("draft",)), (self.st_ver, 4, ("global", "swa"))):
                st.fill(self._pack([], nq, kinds, pad_groups_to=bucket))
                st.upload()
            self._spec_fn(bucket)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _capture(self, body: Callable) -> Callable:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            body()                       # warm-up outside capture (lazy library init)
        torch.cuda.current_stream().wait_stream(s)
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.graph_pool):
            body()
        return g.replay

    # ------------------------------------------------------------------------------------------ speculative
    # EAGLE-style greedy speculation with a one-layer draft head (`speculative/` in the reference; semantics of a
    # top-1 chain, where the tree mask equals the causal mask, `attention/verify-splitk/gemma31_verify.py:19-24`).
    # Per request, with L tokens in the target KV and pending token x_L:
    #   1. draft extend over positions [ld, L] (tokens x_ld..x_L, inputs = target hiddens h_{ld-1}..h_{L-1}): makes the
    #      draft KV exact up to L and proposes d1;
    #   2. two draft decodes (inputs = the draft's own hidden) propose d2, d3;
    #   3. target verify of [x_L, d1, d2, d3] at positions L..L+3 through the split-K verify kernel (n_q = 4);
    #   4. accept the longest prefix with d_{i+1} == argmax_i, plus the target's next token.
    # The whole device part is one CUDA graph per batch bucket; the host sends positions / slots / ids and reads back
    # 7 ints per request.

    def _init_spec(self) -> None:
        h = self.cfg.hidden
        nmax = self.max_running + 1
        self.hbuf = torch.zeros(nmax, 4, h, dtype=torch.bfloat16, device=self.device)
        kinds_d = ("draft",)
        self.st_ext = StagingBuffers(self.max_running * 4, self.max_running, kinds_d, self.device)
        self.st_d2 = StagingBuffers(self.max_running, self.max_running, kinds_d, self.device)
        self.st_d3 = StagingBuffers(self.max_running, self.max_running, kinds_d, self.device)
        self.st_ver = StagingBuffers(self.max_running * 4, self.max_running, ("global", "swa"), self.device)
        self.spec_out = torch.zeros(self.max_running, 7, dtype=torch.int32, device=self.device)
        pin = self.device.type == "cuda"
        self.spec_out_host = torch.zeros(self.max_running, 7, dtype=torch.int32, pin_memory=pin)
        self.dec_resid = torch.zeros(max(self.ecfg.graph_sizes() + [self.max_running]), h, dtype=torch.bfloat16,
                                     device=self.device)
        # scripted drafts (benchmarks with a controlled acceptance rate): per request row, 3 tokens and a mask; a
        # masked-in draft token replaces the draft head's proposal just before verification
        nb = max(self.ecfg.graph_sizes() + [self.max_running])
        self.script_tok = torch.zeros(nb, 3, dtype=torch.int32, device=self.device)
        self.script_mask = torch.zeros(nb, 3, dtype=torch.bool, device=self.device)
        self.script_host = torch.zeros(nb, 4, dtype=torch.int32, pin_memory=pin)
        self.draft_script = None          # callable(request, L) -> [(token, use)] x 3, or None (the draft head alone)

    def _draft_prefill(self, batch: Batch, p: Packed, resid: torch.Tensor, st: StepTensors) -> None:
        """Fill the draft layer's KV over each prefill segment: draft input at position q is (token q, target hidden
        at q - 1); the first position of a segment reuses its own hidden (no earlier hidden in this batch)."""
        shift = torch.arange(len(p.ids), device=self.device) - 1
        shift.clamp_(min=0)
        for s, r0 in p.seg_rows:
            shift[r0] = r0
        self._draft_forward(st, resid[shift])

    def _draft_forward(self, st: StepTensors, hprev: torch.Tensor) -> tuple:
        d = self.draft
        emb = B.embed(st.ids, self.model.embed, self.model.embed_scale)
        x0 = torch.nn.functional.linear(torch.cat([emb, hprev], dim=-1), d.fc)
        st_d = StepTensors(st.ids, st.pos, {"draft": st.slot["draft"]}, st.kv_len, st.req_idx, st.n_q,
                           {"draft": st.splits.get("draft")}, st.ext_segs, st.ext_cache)
        return d.forward(st_d, self.kv, layer_offset=self.cfg.num_layers, inputs_embeds=x0)

    def _draft_logits_argmax(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return self._greedy(x, out)

    def _spec_body(self, bucket: int) -> Callable:
        sp = self._splits(bucket)
        st_ext = self.st_ext.step_tensors(bucket * 4, bucket, 4, sp)
        st_d2 = self.st_d2.step_tensors(bucket, bucket, 1, sp)
        st_d3 = self.st_d3.step_tensors(bucket, bucket, 1, sp)
        st_ver = self.st_ver.step_tensors(bucket * 4, bucket, 4, sp)
        h = self.cfg.hidden
        rows = torch.arange(bucket, device=self.device) * 4
        d_tok = torch.zeros(3, bucket, dtype=torch.int32, device=self.device)
        scripted = self.draft_script is not None            # fixed when the graph is captured
        t_tok = torch.zeros(bucket * 4, dtype=torch.int32, device=self.device)

        def body():
            rix = st_ver.req_idx.long()
            # 1. draft extend: hidden inputs are the stored target hiddens of the request
            hin = self.hbuf[rix].reshape(bucket * 4, h)
            x, resid = self._draft_forward(st_ext, hin)
            sel = rows + (st_ver.pos.view(bucket, 4)[:, 0] - st_ext.pos.view(bucket, 4)[:, 0]).long()
            self._greedy(x[sel], d_tok[0])
            g = resid[sel]
            # 2-3. draft decodes
            for k, stk in ((1, st_d2), (2, st_d3)):
                stk.ids.copy_(d_tok[k - 1])
                x, g = self._draft_forward(stk, g)
                self._greedy(x, d_tok[k])
            if scripted:                                         # controlled acceptance (benchmarks)
                d_tok.copy_(torch.where(self.script_mask[:bucket].t(), self.script_tok[:bucket].t(), d_tok))
            # 4. verify [x_L, d1, d2, d3]
            ids4 = st_ver.ids.view(bucket, 4)
            ids4[:, 1:].copy_(d_tok.t())
            xv, rv = self._target(st_ver)
            self._greedy(xv, t_tok)
            self.hbuf.index_copy_(0, rix, rv.view(bucket, 4, h))
            self.spec_out[:bucket, :4].copy_(t_tok.view(bucket, 4))
            self.spec_out[:bucket, 4:].copy_(d_tok.t())
        return body

    def _spec_fn(self, bucket: int) -> Callable:
        key = ("spec", bucket)
        if key not in self.graphs:
            body = self._spec_body(bucket)
            self.graphs[key] = self._capture(body) if (self.ecfg.cuda_graphs and self.device.type == "cuda") else body
        return self.graphs[key]

    def spec_decode(self, reqs: list) -> dict:
        if not hasattr(self, "hbuf"):
            self._init_spec()
        bucket = self._bucket(len(reqs))
        ext, d2, d3, ver = [], [], [], []
        for r in reqs:
            L = r.kv_len
            ld = r.draft_state.get("ld", L)
            hist = (r.prompt + r.output)
            toks = [hist[p] for p in range(ld, L)] + [r.pending]        # x_ld .. x_L
            ext.append(Segment(r, ld, toks, False))
            d2.append(Segment(r, L + 1, [0], False))
            d3.append(Segment(r, L + 2, [0], False))
            ver.append(Segment(r, L, [r.pending, 0, 0, 0], False))
        for st, segs, nq, kinds in ((self.st_ext, ext, 4, ("draft",)), (self.st_d2, d2, 1, ("draft",)),
                                    (self.st_d3, d3, 1, ("draft",)), (self.st_ver, ver, 4, ("global", "swa"))):
            st.fill(self._pack(segs, nq, kinds, pad_groups_to=bucket))
        self.kv.sync_tables()
        for st in (self.st_ext, self.st_d2, self.st_d3, self.st_ver):
            st.upload()
        if self.draft_script is not None:
            rows = [[0, 0, 0, 0] for _ in range(bucket)]
            for i, r in enumerate(reqs):
                for k, (tok, use) in enumerate(self.draft_script(r, r.kv_len)):
                    rows[i][k] = int(tok)
                    rows[i][3] |= int(bool(use)) << k
            hs = self.script_host[:bucket]
            hs.copy_(torch.tensor(rows, dtype=torch.int32))
            dev_rows = hs.to(self.device, non_blocking=True)
            self.script_tok[:bucket].copy_(dev_rows[:, :3])
            self.script_mask[:bucket].copy_((dev_rows[:, 3:4] >> torch.arange(3, device=self.device)) & 1 == 1)
        self._timed(self._spec_fn(bucket))
        n = len(reqs)
        self.spec_out_host[:n].copy_(self.spec_out[:n], non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        res = {}
        for i, r in enumerate(reqs):
            o = self.spec_out_host[i].tolist()
            t, d = o[:4], o[4:]
            a = 0
            while a < 3 and d[a] == t[a]:
                a += 1
            res[r.rid] = d[:a] + [t[a]]
            r.accepted += a
            r.spec_steps += 1
            r.draft_state["ld"] = r.kv_len + 1                  # draft KV exact up to L after this step's extend
            # hidden rows 0..a of this verify are the next extend's inputs (stored by the graph)
            pg = self.pages.get(r.rid)
            if pg is not None:
                pg["swa"].trim(r.kv_len + a + 1)                  # next target query position L'
                pg["draft"].trim(r.kv_len + 1)                    # next draft extend starts at L + 1
        return res

    def after_synthetic(self, reqs: list) -> None:
        """Synthetic sessions: the draft KV counts as exact up to the prompt end; random target hiddens."""
        if self.spec:
            if not hasattr(self, "hbuf"):
                self._init_spec()
            for r in reqs:
                r.draft_state["ld"] = r.kv_len
            self.hbuf.normal_()
