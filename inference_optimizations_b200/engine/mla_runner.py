"""Model runner for the MLA + DSA + MoE family (`models/mla.py`): paged latent + index pools sharing one page table,
chunked prefill and decode through the same forward (sparse attention makes every prompt token an independent
query over its causal prefix), greedy sampling.  Prefill runs eagerly; decode steps replay a CUDA graph per batch
bucket: the step inputs (token, position, pool slot, visible length, page-table row per request) live in one static
device tensor filled by one pinned host->device copy, padding entries point at the dummy page-table row (page 0,
slot -1: nothing written), and every kernel on the path reads its counts from device memory (expert offsets, top-k
rows), so the MoE's data-dependent grouping needs no host round trip.  Same runner contract as
`engine/runner.py GQARunner` (prefill / decode / attach / detach / can_admit)."""
from __future__ import annotations

from typing import Optional

import torch

from ..config import EngineConfig, MLAMoEConfig
from ..kv.allocator import RequestPages
from ..models.mla import MLAKVCache, MLAModel, MLAStep
from ..ops import basic as B
from ..ops import formats as M_FMT
from ..ops import kvcache as K_OPS
from ..ops.kvcache import FMT_BF16, FMT_FP8, FMT_NVFP4
from .scheduler import Batch, Request, SamplingParams, Segment
from ..ops.formats import INDEX_ROW_BYTES
from ..ops.mla import ROW_BYTES as M_ROW_BYTES


def pool_pages(ecfg: EngineConfig, need: int, page_bytes: int, device) -> int:
    """KV pool size in 64-token pages: what `max_running` requests of `max_seq` need, bounded by
    `max_total_tokens` when set, else by `mem_fraction` of the device memory still free at boot (less a reserve for
    activations) -- the pool never claims memory the weights or the forward need."""
    if ecfg.page_size != 64:
        raise ValueError("KV pools use 64-token pages (page_size must be 64)")
    if ecfg.max_total_tokens > 0:
        return max(3, min(need, ecfg.max_total_tokens // 64 + 2))
    if torch.device(device).type == "cuda":
        free, _total = torch.cuda.mem_get_info(torch.device(device))
        fit = int(max(0, free - (8 << 30)) * ecfg.mem_fraction) // max(1, page_bytes)
        return max(3, min(need, fit))
    return need


def pool_capacity(runner) -> dict:
    """KV-pool capacity at boot on this device for this runner's model: the memory free after the weights (plus what
    the runner's own pools took) sized the way `pool_pages` sizes a memory-bound pool (`mem_fraction` of it, less the
    8 GB activation reserve), in tokens for the NVFP4 352-byte and the FP8 576-byte latent rows (+ the 132-byte index
    key each, every layer)."""
    from ..ops.formats import INDEX_ROW_BYTES
    from ..ops.mla import FMT_FP8, FMT_NVFP4, ROW_BYTES
    kv = runner.kv
    own = sum(t.numel() for t in kv.latent + kv.index + (getattr(kv, "latent4", None) or []))
    free, _ = torch.cuda.mem_get_info(runner.device)
    avail = max(0, free + own - (8 << 30)) * runner.ecfg.mem_fraction
    layers = runner.cfg.num_layers
    tok = {name: int(avail // (layers * (ROW_BYTES[f] + INDEX_ROW_BYTES)))
           for name, f in (("nvfp4", FMT_NVFP4), ("fp8", FMT_FP8))}
    return {"tokens_nvfp4": tok["nvfp4"], "tokens_fp8": tok["fp8"],
            "ratio_nvfp4_vs_fp8": round(tok["nvfp4"] / max(1, tok["fp8"]), 3),
            "note": "latent + index-key bytes of every layer per token, in the memory free at boot after the weights"}


class MLARunner:
    def __init__(self, cfg: MLAMoEConfig, ecfg: EngineConfig, device, max_seq: int, tp_rank: int = 0, tp: int = 1,
                 ep_rank: int = 0, ep_group=None, dcp_rank: int = 0, dcp_group=None, kv_storage=None):
        """ecfg.ep > 1: data-parallel attention + expert-parallel MoE.  Every rank runs its own requests (its own
        scheduler, pools and replicated attention weights); every MoE layer is an exchange over `ep_group` with
        `ecfg.ep` ranks, so all ranks step in lockstep: before each forward the ranks agree on the largest token
        count of the step (one small all-reduce), and a rank without work joins the exchanges with no tokens
        (`idle_step`)."""
        if tp != 1:
            raise NotImplementedError("the MLA family runs attention data-parallel here (tp = 1 per rank)")
        self.cfg, self.ecfg, self.device = cfg, ecfg, torch.device(device)
        self.tp, self.tp_rank = tp, tp_rank
        self.max_seq = max_seq
        self.spec = bool(ecfg.spec) and cfg.draft_layers >= 1
        self.ep_world, self.ep_rank, self.ep_group = max(1, ecfg.ep), ep_rank, ep_group
        # decode context parallelism (ecfg.dcp ranks, every rank runs the same requests): KV sharded by position
        self.dcp_world, self.dcp_rank = max(1, ecfg.dcp), dcp_rank
        if self.dcp_world > 1 and (self.spec or self.ep_world > 1):
            raise NotImplementedError("decode context parallelism runs without speculation or expert parallelism")
        src = None
        if ecfg.checkpoint:                          # HuggingFace DeepSeek-V3-layout checkpoint (this rank's experts)
            from ..models.mla_loader import HFMLASource
            src = HFMLASource(ecfg.checkpoint, cfg, self.device)
        self.model = MLAModel(cfg, self.device, ecfg.seed, ep_rank=ep_rank, ep_world=self.ep_world,
                              dcp_rank=dcp_rank, dcp_world=self.dcp_world, source=src)
        if self.dcp_world > 1:
            self.model.attach_dcp(dcp_group, max(2 * ecfg.max_running, ecfg.chunked_prefill))
        if self.spec:
            self.model.build_draft(ecfg.seed)
        if src is not None:
            src.close()
        if self.ep_world > 1:
            # tokens per exchange: a decode step of every running request (with its draft), or a prefill piece
            self.ep_T_max = max(2 * ecfg.max_running, min(ecfg.chunked_prefill, 1024))
            self.model.attach_ep(ep_group, self.ep_T_max)
        self.mixed = ecfg.kv_dtype == "kvmix"
        if self.mixed and (self.dcp_world > 1 or kv_storage is not None):
            raise NotImplementedError("kvmix pools run without context parallelism or placed pools")
        fmts = {"nvfp4": FMT_NVFP4, "fp8": FMT_FP8, "kvmix": FMT_FP8, "bf16": FMT_BF16}
        if ecfg.kv_dtype not in fmts:
            raise ValueError(f"MLA latent pools hold nvfp4, fp8, kvmix or bf16 rows, not {ecfg.kv_dtype!r}")
        fmt = fmts[ecfg.kv_dtype]
        # bf16: unquantized 1152-byte rows, the accuracy reference of the quantized pools; no kernel reads them, so the
        # attention block runs its torch form (separate writers, fp32 attention) and decode steps are not graphed
        self.ref_pool = fmt == FMT_BF16
        if self.ref_pool:
            if self.dcp_world > 1 or kv_storage is not None:
                raise NotImplementedError("the bf16 reference pool runs without context parallelism or placed pools")
            self.model.fuse_glue = False
        self.max_running = ecfg.max_running
        per_req = (max_seq + 64 + 63) // 64 + 1
        n_layers = cfg.num_layers + int(self.spec)
        pages = pool_pages(ecfg, self.max_running * per_req + 2,
                           n_layers * 64 * (M_ROW_BYTES[fmt] + INDEX_ROW_BYTES), self.device)
        mix = None
        if self.mixed:
            # the byte budget of `pages` FP8 pages, split between FP8 and NVFP4 pages by kvmix_fp8_share
            b8 = n_layers * 64 * (M_ROW_BYTES[FMT_FP8] + INDEX_ROW_BYTES)
            b4 = n_layers * 64 * (M_ROW_BYTES[FMT_NVFP4] + INDEX_ROW_BYTES)
            budget = pages * b8
            p8 = max(2, int(budget * ecfg.kvmix_fp8_share) // b8)
            p4 = max(1, int(budget * (1 - ecfg.kvmix_fp8_share)) // b4)
            mix, pages = (p8, p4, ecfg.kvmix_threshold), p8 + p4
        self.kv = MLAKVCache(cfg, self.device, fmt, self.max_running + 1, per_req, pages,
                             extra_layers=1 if self.spec else 0, latent_div=self.dcp_world, storage=kv_storage,
                             mix=mix)
        self.placement: dict = {}                     # kvmix: rid -> pool chosen at admission ("fp8" | "nvfp4")
        self.promotions = 0
        pages = self.kv.pages
        self.pool_tokens = 64 * (pages - 2)           # KV positions the pool holds (the boot-time capacity)
        self.dummy_row = self.max_running
        self.pages: dict[int, RequestPages] = {}
        self.graphs: dict = {}
        self.graph_launches: dict = {}
        self.event_log = None
        self.prefix_cache = None
        # hybrid models: a cached prefix's pages hold no KDA recurrent state, so their prefixes are reused only with
        # the state cache on (`kda_state_cache`: each request's state is snapshotted whenever its processed length
        # reaches a page boundary, the latest snapshot goes to the prefix's radix node when the request leaves, and
        # a match is cut back to the deepest node holding a state, which is restored into the new request's row).
        # kvmix pools do not reuse prefixes (a promotion would move pages other requests share).
        self.state_fmt = ecfg.kda_state_cache if cfg.kda_every else ""
        if self.state_fmt not in ("", "fp32", "bf16", "fp8"):
            raise ValueError(f"kda_state_cache keeps fp32, bf16 or fp8 state rows, not {self.state_fmt!r}")
        self.snaps: dict = {}                         # rid -> (tokens covered, state snapshot) at a page boundary
        self.state_hits = 0
        if ecfg.prefix_cache and not self.mixed and (not cfg.kda_every or self.state_fmt):
            from ..kv.radix import RadixCache
            self.prefix_cache = RadixCache(self.kv.alloc)

    # ------------------------------------------------------------------------------------------ memory
    def can_admit(self, r: Request) -> bool:
        need = (r.prompt_len + r.params.max_new_tokens + 64) // 64 + 1
        if self.mixed:
            return self._place(r, need)
        reserved = sum(max(0, rp.high_pages - len(rp.pages)) for rp in self.pages.values())
        short = need + reserved - self.kv.alloc.free
        if short > 0 and self.prefix_cache is not None:
            self.prefix_cache.evict(short)
            short = need + reserved - self.kv.alloc.free
        return short <= 0

    def _place(self, r: Request, need: int) -> bool:
        """kvmix admission: the request's pool -- NVFP4 when its length reaches the threshold, else FP8 -- or the
        other pool when the preferred one cannot hold its whole budget (cross-pool fallback); every page of the
        request then comes from that pool."""
        space = self.kv.alloc
        first = space.mix.preferred(r.prompt_len + r.params.max_new_tokens)
        for fmt in (first, "nvfp4" if first == "fp8" else "fp8"):
            reserved = sum(max(0, rp.high_pages - len(rp.pages)) for rp in self.pages.values()
                           if getattr(rp, "fmt", None) == fmt)
            if space.free_in(fmt) - reserved >= need:
                if fmt != first:
                    space.mix.fallbacks += 1
                self.placement[r.rid] = fmt
                return True
        return False

    def attach(self, r: Request) -> None:
        if self.kv.kda:
            self.kv.reset_state(r.slot)         # a new request starts from zero recurrent state
        if self.mixed:
            fmt = self.placement.get(r.rid) or self.kv.alloc.mix.preferred(r.prompt_len + r.params.max_new_tokens)
            rp = RequestPages(self.kv.alloc.view(fmt), self.kv.table, r.slot)
            rp.fmt = fmt
            rp.high_pages = (r.prompt_len + r.params.max_new_tokens + 64) // 64 + 1
            rp.cached = []
            self.pages[r.rid] = rp
            return
        rp = RequestPages(self.kv.alloc, self.kv.table, r.slot)
        rp.high_pages = (r.prompt_len + r.params.max_new_tokens + 64) // 64 + 1
        rp.cached = []
        self.pages[r.rid] = rp

    def on_admit(self, r: Request) -> None:
        """Reuse the longest cached page-aligned prefix of the prompt (at least one prompt token stays to prefill,
        it produces the first output's logits)."""
        self.attach(r)
        if self.prefix_cache is None:
            return
        path = self.prefix_cache.match(r.prompt[: ((r.prompt_len - 1) // 64) * 64])
        if self.state_fmt:                      # hybrid model: reuse only up to the deepest stored recurrent state
            j = max((k for k, n in enumerate(path) if n.state is not None), default=-1)
            self.prefix_cache.release(path[j + 1:])
            path = path[:j + 1]
            if path:
                self.kv.restore_state(r.slot, path[-1].state, self.state_fmt)
                self.state_hits += 1
        rp = self.pages[r.rid]
        for lp, node in enumerate(path):
            rp.pages[lp] = node.page
            self.kv.table.set(r.slot, lp, node.page)
        rp.high = len(path)
        rp.cached = path
        r.prefilled = r.kv_len = r.cached_tokens = 64 * len(path)

    def detach(self, r: Request) -> None:
        rp = self.pages.pop(r.rid, None)
        self.placement.pop(r.rid, None)
        snap = self.snaps.pop(r.rid, None)
        if rp is None:
            return
        if self.prefix_cache is None:
            rp.free()
            return
        hist = (r.prompt + r.output)[: r.kv_len]
        full = len(hist) // 64
        cached = {n.page for n in rp.cached}
        donate = [rp.pages[lp] for lp in range(full)]
        rejected = set(self.prefix_cache.insert(hist[: 64 * full], donate))
        if snap is not None and 0 < snap[0] <= 64 * full:
            nodes = self.prefix_cache.path(hist[: snap[0]])
            if len(nodes) == snap[0] // 64 and nodes[-1].state is None:
                self.prefix_cache.set_state(nodes[-1], snap[1])
                self._trim_states()
        self.prefix_cache.release(rp.cached)
        keep = set(donate) - rejected
        self.kv.alloc.release([pg for pg in rp.pages.values() if pg not in keep and pg not in cached])
        rp.pages.clear()
        self.kv.table.clear(r.slot)

    def _trim_states(self) -> None:
        """Keep at most `kda_state_cache_max` recurrent-state snapshots in the prefix cache, least recent dropped."""
        extra = len(self.prefix_cache.stateful) - max(1, self.ecfg.kda_state_cache_max)
        if extra <= 0:
            return
        nodes = self.prefix_cache.states()
        for n in sorted(nodes, key=lambda n: n.last)[:max(0, extra)]:
            self.prefix_cache.set_state(n, None)

    def _snapshot(self, pairs) -> None:
        """Hybrid models with the state cache: (request, tokens its state now covers) after a forward; a request
        whose processed length sits on a page boundary keeps a snapshot of its recurrent state there."""
        if not self.state_fmt:
            return
        for r, n in pairs:
            if n > 0 and n % 64 == 0:
                self.snaps[r.rid] = (n, self.kv.snapshot_state(r.slot, self.state_fmt))

    # ------------------------------------------------------------------------------------------ lockstep (EP)
    def _agree(self, tokens: int) -> int:
        """Largest token count of this step over the expert-parallel ranks; sets the exchanges per MoE layer."""
        if self.ep_world == 1:
            return tokens
        import torch.distributed as dist
        dev = self.device if dist.get_backend(self.ep_group) == "nccl" else torch.device("cpu")
        v = torch.tensor([tokens], dtype=torch.int64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX, group=self.ep_group)
        m = int(v.item())
        self.model.ep_pieces = max(1, -(-m // self.ep_T_max))
        return m

    def idle_step(self) -> None:
        """A rank without a batch this step: join every exchange the busy ranks run (target MoE layers, then the
        draft layer when speculating), with no tokens."""
        if self.ep_world == 1 or self._agree(0) == 0:
            return
        self.model.ep_idle(self.model.moe_layers())

    # ------------------------------------------------------------------------------------------ steps
    def _step(self, segs: list, agreed: bool = False) -> tuple[MLAStep, list]:
        ids, pos, slot, limit, rix, logit_rows, psel, kseg = [], [], [], [], [], [], [], []
        if self.mixed:
            self._promote([s.req for s in segs], {s.req.rid: s.start + len(s.tokens) for s in segs})
        for s in segs:
            rp = self.pages[s.req.rid]
            rp.ensure(s.start + len(s.tokens))
            if self.mixed:
                psel += [int(rp.fmt == "nvfp4")] * len(s.tokens)
            kseg.append((len(ids), len(s.tokens), s.req.slot))
            for j, tok in enumerate(s.tokens):
                p = s.start + j
                ids.append(int(tok))
                pos.append(p)
                slot.append(rp.slot_of(p))
                limit.append(p + 1)
                rix.append(s.req.slot)
            if s.logits:
                logit_rows.append(len(ids) - 1)
        self.kv.table.sync()
        if self.ecfg.bounds_check:
            from ..tooling.bounds import check_mla_step
            check_mla_step(ids, pos, slot, limit, rix, self.kv, self.max_running + 1, self.cfg.vocab)
        dev = self.device
        mk = lambda v: torch.tensor(v, dtype=torch.int32).to(dev, non_blocking=True)  # noqa: E731
        st = MLAStep(mk(ids), mk(pos), mk(slot), mk(limit), mk(rix), self.max_seq + 1,
                     pool_sel=mk(psel) if self.mixed else None, segs=kseg if self.cfg.kda_every else None)
        if not agreed:
            self._agree(len(ids))
        return st, logit_rows

    def _promote(self, reqs: list, new_len: dict) -> None:
        """kvmix promotion: a request in the FP8 pool whose length reaches the threshold moves to NVFP4 -- fresh
        NVFP4 pages for all its pages, every layer's latent rows re-quantized FP8 -> NVFP4 through the pool writer, its
        index-key pages copied, the page table re-pointed, the FP8 pages freed (stream-ordered before the step that
        reads them).  Without NVFP4 room for the request's whole budget it stays in FP8."""
        space = self.kv.alloc
        thr = space.mix.threshold
        for r in reqs:
            rp = self.pages[r.rid]
            if rp.fmt != "fp8" or new_len[r.rid] < thr or not rp.pages:
                continue
            reserved = sum(max(0, q.high_pages - len(q.pages)) for q in self.pages.values()
                           if getattr(q, "fmt", None) == "nvfp4")
            if space.free_in("nvfp4") - reserved < rp.high_pages:
                continue
            lps = sorted(rp.pages)
            old = [rp.pages[lp] for lp in lps]
            new = space.mix.alloc(len(lps), "nvfp4", fallback=False)
            n_tok = rp.length
            dev = self.device
            src = torch.tensor(old, dtype=torch.long, device=dev)
            dst = torch.tensor(new, dtype=torch.long, device=dev)
            rows = (src[:, None] * 64 + torch.arange(64, device=dev)).reshape(-1)
            drow = ((dst - space.mix.P8)[:, None] * 64 + torch.arange(64, device=dev)).reshape(-1)
            keep = torch.arange(rows.numel(), device=dev) < n_tok        # positions written so far
            for i in range(len(self.kv.latent)):
                # E4M3 values are exact in bf16, the writer kernel's input type
                lat = M_FMT.mla_fp8_row_dequantize(self.kv.latent[i][rows[keep]]).to(torch.bfloat16)
                K_OPS.mla_write(lat[:, :512].contiguous(), lat[:, 512:].contiguous(), drow[keep].int(),
                                self.kv.latent4[i])
                self.kv.index[i][dst] = self.kv.index[i][src]
            for lp, pg in zip(lps, new):
                rp.pages[lp] = pg
                self.kv.table.set(r.slot, lp, pg)
            space.release(old)
            rp.alloc = space.view("nvfp4")
            rp.fmt = "nvfp4"
            self.placement[r.rid] = "nvfp4"
            self.promotions += 1

    def _run(self, segs: list, agreed: bool = False) -> list:
        st, rows = self._step(segs, agreed)

        def body():
            x = self.model.forward(st, self.kv)
            if rows:
                sel = x[torch.tensor(rows, dtype=torch.long, device=self.device)]
                self._out = B.argmax(self.model.logits(sel))
        if self.event_log is not None and self.device.type == "cuda":
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            body()
            e1.record()
            self.event_log.append((e0, e1))
        else:
            body()
        return self._out.cpu().tolist() if rows else []

    def prefill(self, batch: Batch) -> dict:
        for s in batch.segments:
            if s.req.rid not in self.pages:
                self.attach(s.req)
        if self.spec:
            return self._prefill_spec(batch.segments)
        out = self._run(batch.segments)
        self._snapshot((s.req, s.start + len(s.tokens)) for s in batch.segments)
        res, k = {}, 0
        for s in batch.segments:
            if s.logits:
                res[s.req.rid] = int(out[k])
                k += 1
        return res

    # ------------------------------------------------------------------------------------------ split prefill
    # The prefill lane of the SM-partitioned lanes (`engine/pdmux.py`): a prefill batch runs by layer ranges on its
    # own stream while decode graphs replay on the decode lane.  Its launches use the lane's own scratch buffers
    # (`moe_gemm.LANE`), so a chunk the size of a decode batch never shares one with it.
    def split_begin(self, batch: Batch) -> dict:
        if self.spec or self.ep_world > 1 or self.dcp_world > 1:
            raise NotImplementedError("split prefill lanes: speculation, expert / context parallelism not supported")
        for s in batch.segments:
            if s.req.rid not in self.pages:
                self.attach(s.req)
        st, rows = self._step(batch.segments)
        return {"batch": batch, "st": st, "rows": rows, "x": None, "h": None, "x8": None, "index": 0}

    def split_layers(self, sp: dict, count: int) -> bool:
        """Enqueue target layers [index, index + count) of the split on the current stream; after the last layer also
        the LM head and argmax of the rows that want a token (copied to pinned host memory without a wait).  Returns
        True when the split's device work is all enqueued."""
        from ..ops import moe_gemm as MG
        MG.LANE[0] = 1
        try:
            n = self.model.n_target
            lo = sp["index"]
            hi = min(lo + max(1, count), n)
            sp["x"], sp["h"], sp["x8"] = self.model.forward_layers(sp["st"], self.kv, lo, hi, sp["x"], sp["h"],
                                                                   sp["x8"])
            sp["index"] = hi
            if hi < n:
                return False
            if sp["rows"]:
                rows = torch.tensor(sp["rows"], dtype=torch.long)
                rows = rows.pin_memory().to(self.device, non_blocking=True) if self.device.type == "cuda" else rows
                ids = B.argmax(self.model.logits(sp["x"][rows]))
                host = torch.empty(ids.shape, dtype=ids.dtype, pin_memory=self.device.type == "cuda")
                host.copy_(ids, non_blocking=True)
                sp["out_host"] = host
            sp["x"] = sp["h"] = sp["x8"] = None
            return True
        finally:
            MG.LANE[0] = 0

    def split_finish(self, sp: dict) -> dict:
        """Host side of a finished split, after its stream's work completed: rid -> first generated token."""
        res, k = {}, 0
        out = sp.get("out_host")
        self._snapshot((s.req, s.start + len(s.tokens)) for s in sp["batch"].segments)
        for s in sp["batch"].segments:
            if s.logits:
                res[s.req.rid] = int(out[k])
                k += 1
        return res

    # ------------------------------------------------------------------------------------------ MTP speculation
    # Depth-1 multi-token prediction (the DeepSeek-V3 MTP draft; the reference's MLA draft models,
    # `speculative/k3-mla-draft`, and frozen-KV MTP no-sync hooks): the draft layer keeps its own KV for every
    # position the target has processed, so a plain decode step also runs it (one layer) and every step leaves a
    # draft for the next.  A speculative step verifies [pending, draft] at positions (P, P + 1) in one target
    # forward, then runs the draft layer over the same two positions with the true next tokens (o0, o1); the next
    # draft is its prediction at P + 1 when the draft was accepted, else at P.  Greedy verification: the emitted
    # tokens are exactly plain greedy decoding's.
    def _mtp_step(self, st: MLAStep, ids: torch.Tensor) -> MLAStep:
        return MLAStep(ids, st.pos, st.slot, st.limit, st.req_idx, st.max_ctx, pool_sel=st.pool_sel)

    def _prefill_spec(self, segs: list) -> dict:
        st, rows = self._step(segs)
        x, h = self.model.forward_hidden(st, self.kv)
        dev = self.device
        nxt = []
        for s in segs:
            for j in range(len(s.tokens)):
                p = s.start + j
                nxt.append(int(s.tokens[j + 1]) if j + 1 < len(s.tokens)
                           else int(s.req.prompt[p + 1]) if p + 1 < s.req.prompt_len else 0)
        ids = torch.tensor(nxt, dtype=torch.int32).to(dev, non_blocking=True)
        res = {}
        if rows:
            rt = torch.tensor(rows, dtype=torch.long).to(dev, non_blocking=True)
            out = B.argmax(self.model.logits(x[rt]))
            ids[rt] = out                                   # t_{i+1} of a prompt's last position: its first output
        xm = self.model.draft_forward(self._mtp_step(st, ids), self.kv, h)
        if rows:
            d = B.argmax(self.model.logits(xm[rt]))
            both = torch.stack([out, d]).cpu()
            k = 0
            for s in segs:
                if s.logits:
                    res[s.req.rid] = int(both[0, k])
                    s.req.draft_state["d"] = int(both[1, k])
                    k += 1
        return res

    def _decode_mtp(self, reqs: list) -> dict:
        """Plain decode step that also advances the draft layer and leaves the next draft."""
        segs = [Segment(r, r.kv_len, [r.pending], True) for r in reqs]
        st, _ = self._step(segs)
        x, h = self.model.forward_hidden(st, self.kv)
        o = B.argmax(self.model.logits(x))
        d = B.argmax(self.model.logits(self.model.draft_forward(self._mtp_step(st, o), self.kv, h)))
        both = torch.stack([o, d]).cpu()
        for i, r in enumerate(reqs):
            r.draft_state["d"] = int(both[1, i])
        return {r.rid: [int(both[0, i])] for i, r in enumerate(reqs)}

    def spec_decode(self, reqs: list) -> dict:
        segs = [Segment(r, r.kv_len, [r.pending, r.draft_state.get("d", 0)], False) for r in reqs]
        st, _ = self._step(segs)
        # hybrid models: the verify keeps each row's KDA state after its first token (`MLAModel.kda_mid`)
        self.model.kda_mid = {} if self.kv.kda else None
        try:
            x, h = self.model.forward_hidden(st, self.kv)
        finally:
            mid, self.model.kda_mid = self.model.kda_mid, None
        o = B.argmax(self.model.logits(x))                               # [2n]: (o0, o1) per request
        m = B.argmax(self.model.logits(self.model.draft_forward(self._mtp_step(st, o), self.kv, h)))
        both = torch.stack([o, m]).cpu()
        res = {}
        for i, r in enumerate(reqs):
            o0, o1 = int(both[0, 2 * i]), int(both[0, 2 * i + 1])
            acc = o0 == r.draft_state.get("d", -1)
            res[r.rid] = [o0, o1] if acc else [o0]
            r.draft_state["d"] = int(both[1, 2 * i + 1] if acc else both[1, 2 * i])
            r.accepted += int(acc)
            r.spec_steps += 1
            if mid and not acc:                  # rejected draft: the recurrent states advance by the first token only
                for (layer, row), state in mid.items():
                    if row == r.slot:
                        for name, val in state.items():
                            self.kv.kda[layer][name][row].copy_(val)
        self._snapshot((r, r.kv_len + len(res[r.rid])) for r in reqs)
        return res

    def draft_row(self, r: Request) -> int:
        """The draft layer's KV is current after every step (the engine's spec policy prices any step)."""
        return 0

    def decode(self, reqs: list) -> dict:
        if self.spec:
            return self._decode_mtp(reqs)
        bucket = self._bucket(len(reqs))
        agreed = False
        if self.ep_world > 1:
            # expert parallelism: every rank takes part in the same exchanges, so the step's token count is agreed
            # first; a captured graph holds one exchange per MoE layer and replays only when every rank's step fits
            # one (no rank is prefilling a larger piece); graphs are captured collectively (`warm_graphs`), never
            # here, since a capture's warm-up runs exchanges
            self._agree(len(reqs))
            agreed = True
            use_graph = self.model.ep_pieces == 1 and bucket in self.graphs and self._graphable()
        else:
            use_graph = self._graphable() and bucket in self.ecfg.graph_sizes()
        if use_graph:
            out = self._decode_graph(reqs, bucket)
        else:
            segs = [Segment(r, r.kv_len, [r.pending], True) for r in reqs]
            out = self._run(segs, agreed)
        self._snapshot((r, r.kv_len + 1) for r in reqs)
        return {r.rid: [int(out[i])] for i, r in enumerate(reqs)}

    # ------------------------------------------------------------------------------------------ CUDA graphs
    def _bucket(self, n: int) -> int:
        for b in self.ecfg.graph_sizes():
            if b >= n:
                return b
        return n

    def _graphable(self) -> bool:
        """Graphs need every FFN on the block-scaled expert kernels (the bf16 reference MoE path groups tokens on
        the host)."""
        # context parallelism: the merge and reduce kernels pick their buffer half on the host, per call
        return (self.ecfg.cuda_graphs and self.device.type == "cuda" and not self.spec and self.dcp_world == 1
                and not self.ref_pool and all(self.model._quantized_ffn(i) for i in range(self.cfg.num_layers)))

    def _decode_body(self, st: MLAStep, out: torch.Tensor) -> None:
        x = self.model.forward(st, self.kv)
        B.argmax(self.model.logits(x), out=out)

    def _graph(self, bucket: int):
        """(graph, static step tensor [5, bucket] (ids, pos, slot, limit, row), output ids, pinned staging)."""
        if bucket in self.graphs:
            return self.graphs[bucket]
        dev = self.device
        host = torch.zeros(6 if self.mixed else 5, bucket, dtype=torch.int32).pin_memory()
        host[2].fill_(-1)
        host[3].fill_(1)
        host[4].fill_(self.dummy_row)
        step = host.to(dev)
        st = MLAStep(step[0], step[1], step[2], step[3], step[4], self.max_seq + 1,
                     pool_sel=step[5] if self.mixed else None)
        out = torch.zeros(bucket, dtype=torch.int32, device=dev)
        self.model.ep_pieces = 1                # a decode step is one exchange per MoE layer on every rank
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):           # builds the lazily packed experts and workspaces outside capture
            for _ in range(2):
                self._decode_body(st, out)
        torch.cuda.current_stream(dev).wait_stream(side)
        from .._ext import count_launches
        g = torch.cuda.CUDAGraph()
        with count_launches() as cnt, torch.cuda.graph(g):
            self._decode_body(st, out)
        self.graph_launches[bucket] = cnt.n
        self.graphs[bucket] = (g, step, out, host)
        return self.graphs[bucket]

    def _decode_graph(self, reqs: list, bucket: int) -> list:
        g, step, out, host = self._graph(bucket)
        n = len(reqs)
        rows = []
        if self.mixed:
            self._promote(reqs, {r.rid: r.kv_len + 1 for r in reqs})
        for r in reqs:
            rp = self.pages[r.rid]
            p = r.kv_len
            rp.ensure(p + 1)
            row = (int(r.pending), p, rp.slot_of(p), p + 1, r.slot)
            rows.append(row + (int(rp.fmt == "nvfp4"),) if self.mixed else row)
        # one host tensor for the step's inputs (per-element writes into the pinned buffer cost ~1 us each)
        host[:, :n].copy_(torch.tensor(rows, dtype=torch.int32).t())
        if self.mixed:
            host[5, n:] = 0
        host[0, n:] = 0
        host[1, n:] = 0
        host[2, n:] = -1
        host[3, n:] = 1
        host[4, n:] = self.dummy_row
        self.kv.table.sync()
        step.copy_(host, non_blocking=True)
        if self.event_log is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            self.event_log.append((e0, e1))
        else:
            g.replay()
        return out[:n].cpu().tolist()

    @torch.no_grad()
    def score(self, tokens: list) -> torch.Tensor:
        """Teacher-forced full logits [T, V] (fp32, CPU) of one sequence; a scratch request row, freed after."""
        r = Request(rid=-1, prompt=list(tokens), params=SamplingParams(max_new_tokens=1))
        r.slot = next(i for i in range(self.max_running) if all(p.slot != i for p in self.pages.values()))
        self.attach(r)
        try:
            st, _ = self._step([Segment(r, 0, list(tokens), False)])
            return self.model.logits(self.model.forward(st, self.kv)).float().cpu()
        finally:
            self.detach(r)

    def has_graph(self, n: int) -> bool:
        """The decode graph of n's batch bucket is captured."""
        return self._bucket(n) in self.graphs

    def warm_graphs(self, n: int) -> None:
        """Capture the decode graph of the bucket holding n requests (before any timed step).  Under expert
        parallelism this is a collective: every rank calls it at the same point (the capture's warm-up forwards run
        the exchanges)."""
        if self._graphable():
            self._graph(self._bucket(n))

    def count_step_launches(self, bucket: int, kind: Optional[str] = None) -> int:
        """Kernels of this framework in one decode step: the launches issued through the extension while the
        bucket's graph was captured (what every replay runs).  0 when no graph is captured."""
        return self.graph_launches.get(bucket, 0)
