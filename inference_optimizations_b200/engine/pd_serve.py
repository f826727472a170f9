"""In-node prefill / decode disaggregation for the MLA family: one process per GPU, a prefill engine on one GPU and a
decode engine on another, KV pages pushed from the prefill pool straight into the decode pool over NVLink.

The reference runs prefill and decode as separate SGLang servers on disjoint GPUs of one node and replaces the
Mooncake transfer with a one-launch copy over CUDA-IPC-mapped pools (`parallelism/in-node-pd-disaggregation/
pd_nvlink_copy.py:1-30`, `numinous_pdmux_dp.py`).  Here both engines are this framework's `Engine`; the pair shares
one symmetric allocation per pool kind (latent rows, index keys: every layer's pool inside it, `parallel/pd.py
PDPool`), so the prefill side writes into the decode side's pages with plain 16-byte peer stores (`csrc/pd.cu`).

Protocol, one lockstep pass of both ranks (host messages through one object all-gather on a CPU group):
  decode rank   admits new requests while pages last: reserves the prompt's pages in its own allocator (the request
                is attached, its page-table row filled) and sends (request id, prompt, budget, destination pages);
  prefill rank  queues what it received, runs one prefill step; for every prompt that finished, copies the prompt's
                pages of every layer (latent and index pools) into the destination pages, then publishes a sequence
                number in the decode GPU's flag word (stream-ordered after the copies) and sends (request id, first
                token, sequence number); the request's pages are released on the prefill side;
  decode rank   turns each finished prompt into a running request (prompt in the pool, first token pending) after
                enqueueing a bounded device wait for its sequence number on the decode stream -- no host round trip
                sits between the copy and the first decode step -- then runs one decode step.
The pass repeats until every request is done.  Both engines hold the same seeded weights, so the outputs equal a
single engine's (`tests/test_pd_gpu.py`).
"""
from __future__ import annotations

from collections import deque
from typing import Optional

import torch
import torch.distributed as dist

from .engine import Engine
from .scheduler import Request, SamplingParams

PREFILL, DECODE = 0, 1


class PDPair:
    """One side of a prefill / decode pair (role PREFILL = rank 0 of `group`, DECODE = rank 1)."""

    def __init__(self, ecfg, cfg, max_seq: int, group=None, cpu_group=None):
        from ..ops import kvcache as K
        from ..parallel.pd import PDPool
        self.group = group if group is not None else dist.group.WORLD
        self.cpu_group = cpu_group
        self.role = dist.get_rank(self.group)
        if dist.get_world_size(self.group) != 2:
            raise ValueError("a prefill / decode pair is two ranks")
        if ecfg.spec or max(1, ecfg.ep) > 1 or max(1, ecfg.dcp) > 1 or ecfg.prefix_cache:
            raise ValueError("prefill / decode pairs run without speculation, expert / context parallelism and the "
                             "prefix cache")
        if getattr(cfg, "kda_every", 0) or ecfg.kv_dtype == "kvmix":
            raise ValueError("prefill / decode pairs move paged KV only: hybrid KDA models (recurrent states) and "
                             "kvmix pools are not transferred")
        dev = torch.device(ecfg.device)
        self.pools = {}
        # without GPUs (gloo ranks) the pages travel inside the host messages instead of over peer memory: the same
        # protocol, testable on the CPU
        self.host = dev.type != "cuda"

        def storage(layers: int, pages: int, row_bytes: int):
            t = torch.tensor([pages], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.cpu_group)   # one page space on both sides
            pages = int(t.item())
            if self.host:
                lat = [torch.zeros(pages * 64, row_bytes, dtype=torch.uint8) for _ in range(layers)]
                idx = [torch.zeros(pages, K.INDEX_PAGE_BYTES, dtype=torch.uint8) for _ in range(layers)]
                self.pools = {"latent": lat, "index": idx}
                return pages, lat, idx
            lat = PDPool(layers, pages, 64 * row_bytes, dev, group=self.group)
            idx = PDPool(layers, pages, K.INDEX_PAGE_BYTES, dev, group=self.group)
            self.pools = {"latent": lat, "index": idx}
            return (pages, [lat.layer(i).view(pages * 64, row_bytes) for i in range(layers)],
                    [idx.layer(i) for i in range(layers)])
        self.eng = Engine(ecfg, cfg, max_seq=max_seq, kv_storage=storage)
        self.runner = self.eng.runner
        self.seq = 0
        self.inflight: dict[int, Request] = {}       # decode side: pages reserved, prompt not yet arrived
        self.prefill_of: dict[int, tuple] = {}        # prefill side: engine request id -> (pair rid, dst pages)
        self.transfers = 0

    # ------------------------------------------------------------------------------------------ prefill side
    def _push(self, r: Request, dst: list):
        """Copy the prompt's pages of every layer into the decode pool's `dst` pages, then publish a new sequence
        number in the decode GPU's flag (the copies of both pool kinds precede the release on this stream).
        -> the sequence number (host transport: the pages' bytes, for the message)."""
        from .._ext import ext
        rp = self.runner.pages[r.rid]
        n = len(dst)
        if self.host:
            self.transfers += 1
            pg = torch.tensor([rp.pages[lp] for lp in range(n)], dtype=torch.long)
            rows = (pg[:, None] * 64 + torch.arange(64)).reshape(-1)
            return ([t[rows].clone() for t in self.pools["latent"]], [t[pg].clone() for t in self.pools["index"]])
        src = torch.tensor([rp.pages[lp] for lp in range(n)], dtype=torch.int32, device=self.eng.device)
        dpt = torch.tensor(dst, dtype=torch.int32, device=self.eng.device)
        for pool in self.pools.values():
            ext().pd_copy(pool.buf, pool.ptrs[DECODE], src, dpt, pool.page_bytes, pool.layers, pool.layer_stride,
                          pool.layer_stride)
        self.seq += 1
        lat = self.pools["latent"]
        ext().pd_signal(lat.ptrs[DECODE] + lat.flag_off, self.seq, lat.buf)
        self.transfers += 1
        return self.seq

    def _prefill_pass(self, plans: list) -> list:
        for rid, prompt, _budget, dst in plans:
            # this side only produces the first token: a budget of 2 keeps the request alive (not finished, pages
            # held) until its pages are pushed, and reserves no decode pages here
            r = self.eng.add_request(prompt, SamplingParams(max_new_tokens=2))
            self.prefill_of[r.rid] = (rid, dst)
        done = []
        if self.eng.sched.prefilling is not None or self.eng.sched.waiting:
            out = self.eng.step()
            for r in list(self.eng.sched.running):          # prompts that finished this step: hand them over
                if r.rid not in out:
                    continue
                rid, dst = self.prefill_of.pop(r.rid)
                seq = self._push(r, dst)
                done.append((rid, out[r.rid][0], seq))
                self.eng.sched.running.remove(r)
                self.eng.sched.free_slots.append(r.slot)
                r.finished = True
                self.runner.detach(r)
        return done

    # ------------------------------------------------------------------------------------------ decode side
    def _reserve(self, todo: deque) -> list:
        """Admit requests from the front of `todo` while slots and pages last: attach them and reserve their
        prompt pages.  -> plans for the prefill side."""
        sched, plans = self.eng.sched, []
        while todo and sched.free_slots and len(sched.running) + len(self.inflight) < sched.max_running:
            rid, prompt, params = todo[0]
            r = Request(rid, list(prompt), params)
            if not self.runner.can_admit(r):
                break
            todo.popleft()
            r.slot = sched.free_slots.pop()
            self.runner.attach(r)
            rp = self.runner.pages[r.rid]
            rp.ensure(r.prompt_len)
            self.inflight[rid] = r
            dst = [rp.pages[lp] for lp in range(-(-r.prompt_len // 64))]
            plans.append((rid, r.prompt, params.max_new_tokens, dst))
        return plans

    def _arrive(self, done: list) -> None:
        lat = self.pools["latent"]
        sched = self.eng.sched
        for rid, tok, seq in done:
            r = self.inflight.pop(rid)
            if self.host:
                rp = self.runner.pages[rid]
                pg = torch.tensor([rp.pages[lp] for lp in range(-(-r.prompt_len // 64))], dtype=torch.long)
                rows = (pg[:, None] * 64 + torch.arange(64)).reshape(-1)
                for t, v in zip(lat, seq[0]):
                    t[rows] = v
                for t, v in zip(self.pools["index"], seq[1]):
                    t[pg] = v
            else:
                lat.wait(seq)                    # the decode stream waits for the pages (bounded, device-side)
            r.prefilled = r.kv_len = r.prompt_len
            r.pending = tok
            r.output.append(tok)
            sched.running.append(r)
            sched._check_done(r)
            if r.finished:
                self.eng.finished.append(r)
                self.runner.detach(r)

    # ------------------------------------------------------------------------------------------ both
    def serve(self, prompts: Optional[list] = None, params: Optional[SamplingParams] = None) -> list:
        """Run the pair until every prompt is done.  The decode rank passes the prompts and gets their outputs (in
        order); the prefill rank passes nothing and gets an empty list."""
        params = params or SamplingParams()
        todo = deque((i, p, params) for i, p in enumerate(prompts or [])) if self.role == DECODE else deque()
        reqs: dict[int, Request] = {}
        done: list = []
        while True:
            if self.role == DECODE:
                plans = self._reserve(todo)
                for rid, *_ in plans:
                    reqs[rid] = self.inflight[rid]
                busy = bool(todo or self.inflight or self.eng.sched.running)
                msg = {"plans": plans, "busy": busy}
            else:
                msg = {"done": done, "busy": bool(self.prefill_of)}
            both = [None, None]
            dist.all_gather_object(both, msg, group=self.cpu_group)
            if not both[DECODE]["busy"] and not both[PREFILL]["busy"]:
                break
            if self.role == PREFILL:
                done = self._prefill_pass(both[DECODE]["plans"])
            else:
                self._arrive(both[PREFILL]["done"])
                if self.eng.sched.running:
                    self.eng.step()
        if not self.host:
            torch.cuda.synchronize(self.eng.device)
        if self.role == DECODE:
            if not self.host:
                self.pools["latent"].check()
            return [reqs[i].output for i in sorted(reqs)]
        return []
