"""Public serving API: `Engine(EngineConfig).generate(prompts)` or `add_request` + `step()` in a loop.

One Engine per process / GPU.  With tensor parallelism every rank runs the same Engine; rank 0's scheduler decides and
the decision (the packed step inputs) is identical on every rank because every rank receives the same requests in the
same order (the HTTP front end broadcasts them, `server/http.py`), so the per-step host traffic needs no collective.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Optional

import torch

from ..config import EngineConfig, GQAConfig, model_config
from .runner import GQARunner
from .scheduler import Request, SamplingParams, Scheduler
from .spec_policy import SpecPolicy


@dataclass
class StepStats:
    kind: str                     # "prefill" | "decode" | "spec"
    tokens_out: int
    seconds: float


class Engine:
    def __init__(self, ecfg: EngineConfig, model_cfg=None, max_seq: int = 4096, tp_rank: int = 0, tp: int = 1,
                 all_reduce=None, argmax_merge=None, global_pages: Optional[int] = None, ep_rank: int = 0,
                 ep_group=None, dcp_rank: int = 0, dcp_group=None, kv_storage=None):
        """kv_storage (MLA family): places the KV pools (`MLAKVCache(storage=)`; prefill / decode disaggregation)."""
        self.ecfg = ecfg
        self.cfg = model_cfg if model_cfg is not None else model_config(ecfg.model)
        self.device = torch.device(ecfg.device)
        if isinstance(self.cfg, GQAConfig):
            self.runner = GQARunner(self.cfg, ecfg, self.device, max_seq, tp_rank, tp, all_reduce, argmax_merge,
                                    global_pages)
        else:
            from .mla_runner import MLARunner
            self.runner = MLARunner(self.cfg, ecfg, self.device, max_seq, tp_rank, tp, ep_rank, ep_group, dcp_rank,
                                    dcp_group, kv_storage=kv_storage)
        self.sched = Scheduler(ecfg.max_running, ecfg.chunked_prefill, ecfg.decode_burst,
                               can_admit=self.runner.can_admit, on_admit=getattr(self.runner, "on_admit", None))
        self.stats: list[StepStats] = []
        self.finished: list[Request] = []
        self.spec_policy = SpecPolicy(ecfg.draft_tokens, ecfg.spec_policy)
        self.pdmux = None
        if getattr(ecfg, "pdmux", False):
            # the lanes split a GQA prefill by layer ranges on one rank; refuse the combinations that would only fail
            # at the first prefill (inside split_begin), e.g. in the middle of an HTTP serving loop
            bad = [why for cond, why in ((bool(ecfg.spec), "speculative decoding"), (tp > 1, "tp > 1"),
                                         (max(1, ecfg.ep) > 1, "expert parallelism"),
                                         (max(1, ecfg.dcp) > 1, "context parallelism"))
                   if cond]
            if bad:
                raise ValueError("EngineConfig(pdmux=True) does not support " + ", ".join(bad))
            from .pdmux import PdmuxEngine
            self.pdmux = PdmuxEngine(self, token_budget=ecfg.pdmux_budget)
        self.trace = None
        if ecfg.trace:
            from ..tooling.trace import StepTrace
            self.trace = StepTrace(ecfg.trace, tp_rank)

    def has_work(self) -> bool:
        return self.pdmux.has_work() if self.pdmux is not None else self.sched.has_work()

    def add_request(self, prompt: list, params: Optional[SamplingParams] = None) -> Request:
        return self.sched.new_request(prompt, params or SamplingParams())

    def step(self, hold: Optional[bool] = None, chunk_cap: int = 0, park: bool = False) -> dict:
        """One engine iteration.  Returns rid -> tokens produced this step.  hold / chunk_cap / park: the
        data-parallel ranks' joint decode-burst decision, prefill budget and pacing decision for this pass
        (`generate_dp`); default: local rules."""
        if self.pdmux is not None:
            return self._pdmux_step()
        t0 = time.perf_counter()
        rec = self.trace.begin() if self.trace else None
        batch = self.sched.schedule(hold, chunk_cap, park)
        if batch is None:
            if getattr(self.runner, "ep_world", 1) > 1:
                self.runner.idle_step()          # data-parallel attention: join the busy ranks' MoE exchanges
            return {}
        if rec is not None:
            t_s = self.trace.phase(rec, "schedule", t0)
            log = getattr(self.runner, "event_log", None)
            n_ev = len(log) if log is not None else None
            if log is None and self.device.type == "cuda":
                self.runner.event_log = []
                n_ev = 0
        if batch.kind == "prefill":
            nxt = self.runner.prefill(batch)
            self.sched.commit_prefill(batch, nxt)
            out = {rid: [t] for rid, t in nxt.items()}
        else:
            reqs = [s.req for s in batch.segments]
            spec_on = getattr(self.runner, "spec", False)
            kind = "decode"
            if spec_on and self.spec_policy.use_spec(
                    [r.rid for r in reqs], can_spec=not any(r.draft_state.get("stale") for r in reqs),
                    can_price=all(self.runner.draft_row(r) <= 3 for r in reqs)):
                before = sum(r.accepted for r in reqs)
                t1 = time.perf_counter()
                kind = "spec"
                out = self.runner.spec_decode(reqs)
                self.spec_policy.observe_spec((sum(r.accepted for r in reqs) - before) / len(reqs),
                                              time.perf_counter() - t1)
            else:
                t1 = time.perf_counter()
                out = self.runner.decode(reqs)
                if spec_on:
                    self.spec_policy.observe_plain(time.perf_counter() - t1)
            self.sched.commit_decode(out)
        for r in [s.req for s in batch.segments]:
            if r.finished and r not in self.finished:
                self.finished.append(r)
                self.runner.detach(r)
        self.stats.append(StepStats(batch.kind if batch.kind == "prefill" else kind,
                                    sum(len(v) for v in out.values()), time.perf_counter() - t0))
        if rec is not None:
            self.trace.phase(rec, "run+commit", t_s)
            rec.update(kind=self.stats[-1].kind, tokens=self.stats[-1].tokens_out, running=len(self.sched.running),
                       waiting=len(self.sched.waiting), batch=len(batch.segments))
            ev = None
            log = getattr(self.runner, "event_log", None)
            if n_ev is not None and log is not None and len(log) > n_ev:
                ev = log[-1]
                if len(log) > 4096:          # the trace keeps its own reference; bound the runner's list
                    del log[:-1]
            self.trace.end(rec, ev)
        return out

    def _pdmux_step(self) -> dict:
        """One lanes iteration, recorded like any other step (StepStats, trace): kind "prefill" when a split advanced
        this iteration and no decode ran, else "decode"."""
        t0 = time.perf_counter()
        rec = self.trace.begin() if self.trace else None
        n_log = len(self.pdmux.log)
        out = self.pdmux.step()
        kind = "decode"
        if len(self.pdmux.log) > n_log:
            _grp, span, dbs = self.pdmux.log[-1]
            if span is not None and not dbs:
                kind = "prefill"
        self.stats.append(StepStats(kind, sum(len(v) for v in out.values()), time.perf_counter() - t0))
        if rec is not None:
            self.trace.phase(rec, "lanes", t0)
            rec.update(kind=kind, tokens=self.stats[-1].tokens_out, running=len(self.sched.running),
                       waiting=len(self.sched.waiting), batch=0)
            self.trace.end(rec, None)
        return out

    def generate_dp(self, prompts: list, params: Optional[SamplingParams] = None, group=None,
                    route: bool = False) -> list:
        """Data-parallel serving loop.  Every pass the ranks all-gather one row of scheduler facts (waiting, running,
        decode streak, last pass kind, chunked prefill pending, passes delayed, prefill backlog) and take the same
        decisions from it: stop when no rank has work; hold prefill admission everywhere while decode bursts run
        (`burst.dp_hold`: streak below the burst on a decoding rank, queues short, bounded delay); cap every rank's
        prefill at the budget of the ranks' backlogs (`dp_policy.prefill_budget`).  The expert-parallel exchanges
        stay in lockstep since every rank steps once per pass.
        route=False: `prompts` are this rank's; returns their outputs.  route=True: `prompts` is the global list
        (identical on every rank); the cache-aware balancer (`dp_policy.DPBalancer`) assigns each prompt to a rank
        (the same assignment on every rank) and the return value is {global index: output} for this rank's share."""
        import torch.distributed as dist
        from .burst import RankFacts, dp_hold
        from .dp_policy import DPBalancer, pace_decide, prefill_budget, skew_chunk_cap
        if self.pdmux is not None and self.pdmux.group is None:
            raise ValueError("generate_dp with pdmux needs the lanes' CPU group (PdmuxEngine(group=...)): the lanes "
                             "of data-parallel ranks advance in lockstep through it")
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        if route:
            bal = DPBalancer(world)
            mine = [i for i, p in enumerate(prompts) if bal.route(p, t=0.0) == rank]
            reqs = {i: self.add_request(prompts[i], params) for i in mine}
        else:
            reqs = {i: self.add_request(p, params) for i, p in enumerate(prompts)}
        dev = self.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
        delayed = pace_streak = 0
        self.dp_log: list = []
        while True:
            f = self.sched.facts()
            row = torch.tensor(f[:5] + [delayed, f[5], int(self.has_work())], dtype=torch.int64, device=dev)
            parts = [torch.empty_like(row) for _ in range(world)]
            dist.all_gather(parts, row, group=group)
            rows = [p.cpu().tolist() for p in parts]
            if not any(r[7] for r in rows):
                break
            hold = dp_hold([RankFacts.from_row(r[:6]) for r in rows], self.ecfg.decode_burst,
                           self.ecfg.burst_queue_cap, self.ecfg.max_delay_passes)
            cap = prefill_budget([r[6] for r in rows], self.ecfg.chunked_prefill, min_tokens=min(
                2048, self.ecfg.chunked_prefill), page=self.ecfg.page_size)
            park = False
            if self.ecfg.dp_pace_steps > 0:
                # pacing: park lone continuing chunked prefills for a bounded number of passes while other ranks
                # only decode (every rank takes the same decision from the same rows)
                action, pace_streak = pace_decide([r[0] > 0 for r in rows], [r[4] > 0 for r in rows],
                                                  [r[1] for r in rows], [r[0] for r in rows], pace_streak,
                                                  steps=self.ecfg.dp_pace_steps)
                park = action == "park"
            if self.ecfg.dp_skew_floor > 0:
                # skew: a rank extending while the others extend less takes at most max(floor, their largest)
                ext = [min(r[6], self.ecfg.chunked_prefill) if (r[4] or (r[0] and not hold)) else 0 for r in rows]
                sk = skew_chunk_cap(ext[rank], ext[:rank] + ext[rank + 1:], floor=self.ecfg.dp_skew_floor,
                                    page=self.ecfg.page_size)
                cap = min(c for c in (cap, sk) if c > 0) if (cap or sk) else 0
            self.dp_log.append((hold, cap, park))
            self.step(hold=hold, chunk_cap=cap, park=park)
            delayed = delayed + 1 if hold else 0
        if route:
            return {i: r.output for i, r in reqs.items()}
        return [r.output for r in reqs.values()]

    def generate(self, prompts: list, params: Optional[SamplingParams] = None, max_steps: int = 1 << 30) -> list:
        reqs = [self.add_request(p, params) for p in prompts]
        steps = 0
        while self.has_work() and steps < max_steps:
            self.step()
            steps += 1
        return [r.output for r in reqs]
