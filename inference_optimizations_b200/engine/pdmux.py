"""SM-partitioned prefill / decode lanes on one GPU ("pdmux").

A prefill chunk runs as a *split*: a few decoder layers per engine iteration, enqueued on the prefill lane's stream,
while every iteration also runs one decode step of the running requests on the decode lane's stream.  The lanes'
streams belong to green contexts over disjoint SM sets of the GPU (`csrc/lanes.cu`), so a long prefill does not stall
decode for its whole duration and decode keeps a fixed share of the SMs.

Reference behaviour: the pdmux loop and its data-parallel rules (`parallelism/in-node-pd-disaggregation/
numinous_pdmux_dp.py:1-24`, `split_forward_count` :35, `choose_stream_idx` :44), the layer-range split prefill
(`glm_pdmux_split_hooks.py:1-30`) and the three-group configuration (`glm_pdmux/glm_pdmux.yaml:1-11`).

Stream groups: 0 = prefill alone on every SM, n - 1 = decode alone on every SM, 1 .. n - 2 = both lanes on disjoint
partitions whose decode share grows with the index.  Under data parallelism every choice is made from GLOBAL state
(one all-gather of (prefill tokens, decode requests) per iteration on a CPU process group): a split starts on every
rank in the same iteration (an idle split where a rank has no prefill), advances the same layer range and finishes in
the same iteration.

A split whose last layers are enqueued stays pending while decode iterations go on; it is committed (first tokens, the
requests join the decode batch) in the first iteration in which its event has fired on every rank, so neither the host
nor the decode stream ever waits on the prefill lane.
Not supported with the lanes: speculative decoding and tensor parallelism (the runner raises).
"""
from __future__ import annotations

from typing import Optional

import torch

from .scheduler import SamplingParams

SM_GRANULE = 8      # green-context SM partitions on sm_90 and later are multiples of 8 SMs


# ------------------------------------------------------------------------------------------------------ pure rules
def split_layer_count(global_tokens: list, budget: int, num_layers: int, split_index: int) -> int:
    """Decoder layers the split advances this iteration: the token budget over the LARGEST per-rank prefill (at least
    one layer), so every rank runs the same range; with no prefill tokens anywhere (every split idle) the split
    finishes at once."""
    m = max(global_tokens, default=0)
    step = num_layers if m <= 0 else max(1, budget // m)
    return max(0, min(num_layers, split_index + step) - split_index)


def choose_group(n_groups: int, split_active: bool, decode_active: bool, max_decode_bs: int,
                 thresholds: tuple = (), decode_bs_divisor: int = 36) -> int:
    """Stream group for this iteration from global state.  With both lanes busy: the split group whose decode share
    fits the largest decode batch -- the last of the ascending `thresholds` (one per split group) that the batch
    reaches, or proportionally to max_decode_bs / decode_bs_divisor."""
    if n_groups < 3:
        raise ValueError("pdmux needs at least 3 stream groups (prefill-only, one split, decode-only)")
    if not split_active:
        return n_groups - 1 if decode_active else 0
    if not decode_active:
        return 0
    n_split = n_groups - 2
    if thresholds:
        k = 1
        for i, t in enumerate(thresholds[:n_split]):
            if max_decode_bs >= t:
                k = i + 1
        return k
    return 1 + min(n_split - 1, max_decode_bs * n_split // max(1, decode_bs_divisor))


def divide_sms(total: int, n_groups: int, granule: int = SM_GRANULE) -> list:
    """(prefill SMs, decode SMs) per stream group.  Split group k gives decode k / (n - 1) of the SMs, rounded to the
    partition granule; 0 means 'every SM' for the one busy lane of groups 0 and n - 1."""
    out = [(total, 0)]
    for k in range(1, n_groups - 1):
        d = int(round(total * k / (n_groups - 1) / granule)) * granule
        d = min(max(granule, d), total - granule)
        out.append((total - d, d))
    out.append((0, total))
    return out


# ------------------------------------------------------------------------------------------------------ streams
class Lanes:
    """The prefill and decode streams of every stream group on one device.  The all-SM groups use two ordinary
    streams; each split group one pair of green-context streams (created on first use, kept for the process)."""

    def __init__(self, device, n_groups: int = 3, divisions: Optional[list] = None):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        if self.cuda and self.device.index is None:       # a bare "cuda" means the current device, as in torch
            self.device = torch.device("cuda", torch.cuda.current_device())
        total = torch.cuda.get_device_properties(self.device).multi_processor_count if self.cuda else 0
        self.divisions = divisions or divide_sms(total, n_groups)
        self.sms: dict = {}              # group -> (prefill SMs, decode SMs) as the driver partitioned them
        self._streams: dict = {}
        self._full = None

    def streams(self, group: int):
        if not self.cuda:
            return None, None
        if group not in self._streams:
            p_sms, d_sms = self.divisions[group]
            if p_sms == 0 or d_sms == 0:
                if self._full is None:
                    self._full = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
                self._streams[group] = self._full
                self.sms[group] = (p_sms, d_sms)
            else:
                from .._ext import ext
                d_handle, p_handle, d_got, p_got = ext().sm_lanes(self.device.index, d_sms)
                self._streams[group] = (torch.cuda.ExternalStream(p_handle, device=self.device),
                                        torch.cuda.ExternalStream(d_handle, device=self.device))
                self.sms[group] = (p_got, d_got)
        return self._streams[group]


# ------------------------------------------------------------------------------------------------------ the loop
class _StreamCtx:
    def __init__(self, s):
        self.ctx = torch.cuda.stream(s) if s is not None else None

    def __enter__(self):
        if self.ctx is not None:
            self.ctx.__enter__()
        return self

    def __exit__(self, *a):
        if self.ctx is not None:
            self.ctx.__exit__(*a)


class PdmuxEngine:
    """Drives an `Engine` (GQA or MLA family, tp = 1, no speculation, expert or context parallelism) with the
    prefill and decode lanes.

    group: optional CPU (gloo) process group of the data-parallel ranks; every rank then calls `step()` in lockstep
    (`generate` loops until no rank has work)."""

    def __init__(self, engine, n_groups: int = 3, token_budget: int = 65536, decode_bs_divisor: int = 36,
                 thresholds: tuple = (), group=None, divisions: Optional[list] = None):
        self.engine = engine
        self.n_groups = n_groups
        self.budget = token_budget
        self.divisor = decode_bs_divisor
        self.thresholds = tuple(thresholds)
        self.group = group
        self.lanes = Lanes(engine.device, n_groups, divisions)
        model = engine.runner.model
        self.num_layers = getattr(model, "n_target", len(model.layers))
        self.split: Optional[dict] = None
        self.pending: Optional[dict] = None   # a split whose device work is all enqueued, not yet committed
        self._p_event = None
        self._p_stream = None
        self.log: list = []               # per iteration: (group, split layers [lo, hi), decode batch size)

    def _global(self, p_tokens: int, d_reqs: int, work: int) -> tuple:
        if self.group is None:
            return [p_tokens], [d_reqs], work
        import torch.distributed as dist
        mine = torch.tensor([p_tokens, d_reqs, work], dtype=torch.int64)
        allv = [torch.zeros(3, dtype=torch.int64) for _ in range(dist.get_world_size(self.group))]
        dist.all_gather(allv, mine, group=self.group)
        return [int(v[0]) for v in allv], [int(v[1]) for v in allv], max(int(v[2]) for v in allv)

    def step(self) -> dict:
        """One iteration: maybe start a split, advance it by its layer range on the prefill lane, one decode step on
        the decode lane, and commit a split whose device work has completed on every rank.  A split whose last layers
        are enqueued stays pending (decode keeps running) until its event has fired: the host never blocks on the
        prefill lane.  Returns rid -> tokens produced."""
        eng = self.engine
        sched, run = eng.sched, eng.runner
        if self.group is None and self.pending is not None and self.pending.get("event") is not None and \
                not sched.running:
            self.pending["event"].synchronize()      # nothing to decode: waiting on the prefill lane costs nothing
        busy = 1 if (self.pending is not None and self.pending.get("event") is not None
                     and not self.pending["event"].query()) else 0
        batch = sched.plan_prefill() if self.split is None and self.pending is None else None
        if self.split is not None:
            p_tok = self.split["tokens"]
        else:
            p_tok = sum(len(s.tokens) for s in batch.segments) if batch is not None else 0
        dbatch = sched.decode_batch()
        gp, gd, any_busy = self._global(p_tok, len(dbatch.segments) if dbatch is not None else 0, busy)
        split_active = self.split is not None or max(gp) > 0
        lane_busy = split_active or self.pending is not None
        grp = choose_group(self.n_groups, lane_busy, max(gd) > 0, max(gd), self.thresholds, self.divisor)
        ps, ds = self.lanes.streams(grp)
        span = None
        if split_active:
            with _StreamCtx(ps):
                if ps is not None and self._p_event is not None and ps is not self._p_stream:
                    ps.wait_event(self._p_event)          # the split's earlier layers ran on another stream
                if self.split is None:
                    self.split = run.split_begin(batch) if batch is not None else {"idle": True, "index": 0}
                    self.split["tokens"] = p_tok
                count = split_layer_count(gp, self.budget, self.num_layers, self.split["index"])
                lo = self.split["index"]
                if self.split.get("idle"):
                    self.split["index"] = lo + count
                    done = self.split["index"] >= self.num_layers
                else:
                    done = run.split_layers(self.split, count)
                span = (lo, self.split["index"])
                if ps is not None:
                    self._p_event = torch.cuda.Event()
                    self._p_event.record(ps)
                    self._p_stream = ps
            if done:
                self.split["event"] = self._p_event if not self.split.get("idle") else None
                self.pending, self.split = self.split, None
                any_busy = 1                              # committed in a later iteration, on every rank together
        out: dict = {}
        if dbatch is not None:
            reqs = [s.req for s in dbatch.segments]
            if run.device.type == "cuda" and run.ecfg.cuda_graphs and not run.has_graph(len(reqs)):
                run.warm_graphs(len(reqs))
            with _StreamCtx(ds):
                out = run.decode(reqs)
            sched.commit_decode(out)
        finished = None
        if self.pending is not None and not any_busy:
            finished, self.pending = self.pending, None
            if not finished.get("idle"):
                if finished.get("event") is not None:
                    finished["event"].synchronize()      # already complete: no wait
                nxt = run.split_finish(finished)
                sched.commit_prefill(finished["batch"], nxt)
                for rid, t in nxt.items():
                    out.setdefault(rid, []).append(t)
        cand = [sg.req for sg in dbatch.segments] if dbatch is not None else []
        if finished is not None and not finished.get("idle"):
            cand += [sg.req for sg in finished["batch"].segments]
        for r in cand:
            if r.finished and r not in eng.finished:
                eng.finished.append(r)
                run.detach(r)
        self.log.append((grp, span, len(dbatch.segments) if dbatch is not None else 0))
        return out

    def has_work(self) -> bool:
        return self.engine.sched.has_work() or self.split is not None or self.pending is not None

    def generate(self, prompts: list, params: Optional[SamplingParams] = None, max_steps: int = 1 << 30) -> list:
        reqs = [self.engine.add_request(p, params) for p in prompts]
        steps = 0
        while steps < max_steps:
            busy = 1 if self.has_work() else 0
            if self.group is not None:
                busy = self._global(0, 0, busy)[2]
            if not busy:
                break
            self.step()
            steps += 1
        return [r.output for r in reqs]


# ------------------------------------------------------------------------------------------------------ benchmark
def _window(step, eng, prompt: list) -> dict:
    """Inject one long prompt into a running decode batch and step until its first token: time to first token, and
    the decode batch's inter-token gaps and throughput over that window."""
    import time
    r = eng.add_request(prompt, SamplingParams(max_new_tokens=1, ignore_eos=True))
    t0 = last = time.perf_counter()
    gaps, dec = [], 0
    for _ in range(100000):
        if r.output:
            break
        out = step()
        now = time.perf_counter()
        n = sum(len(v) for rid, v in out.items() if rid != r.rid)
        if n:
            gaps.append(now - last)
            last = now
            dec += n
    else:
        raise RuntimeError("the long prompt never produced a token")
    ttft = time.perf_counter() - t0
    return {"ttft_ms": round(ttft * 1e3, 1), "max_gap_ms": round(max(gaps, default=0) * 1e3, 1),
            "mean_gap_ms": round(sum(gaps) / max(1, len(gaps)) * 1e3, 2), "decode_tok_s": round(dec / ttft, 1)}


def main() -> None:
    """Decode batch + one long prefill, plain engine (chunked prefill, decode-burst rule) vs the SM-partitioned lanes:
    python -m inference_optimizations_b200.engine.pdmux --layers 12 --decode 32 --ctx 2048 --prompt 16384"""
    import argparse
    import json
    from dataclasses import replace

    from ..config import EngineConfig, model_config
    from .engine import Engine
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gemma31b")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--decode", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--prompt", type=int, default=16384)
    ap.add_argument("--chunk", type=int, default=8192)
    ap.add_argument("--budget", type=int, default=65536)
    ap.add_argument("--burst", type=int, default=1)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--kv", default="nvfp4")
    ap.add_argument("--groups", type=int, default=3)
    ap.add_argument("--divisor", type=int, default=36)
    a = ap.parse_args()
    cfg = replace(model_config(a.model), num_layers=a.layers)
    res = {"model": a.model, "layers": a.layers, "decode_batch": a.decode, "ctx": a.ctx, "prompt": a.prompt,
           "chunk": a.chunk, "groups": a.groups, "divisor": a.divisor}
    for mode in ("plain", "pdmux"):
        ecfg = EngineConfig(model=a.model, device=a.device, kv_dtype=a.kv, max_running=a.decode + 2,
                            chunked_prefill=a.chunk, decode_burst=a.burst)
        eng = Engine(ecfg, cfg, max_seq=max(a.ctx + 2048, a.prompt) + 1024)
        pm = PdmuxEngine(eng, n_groups=a.groups, token_budget=a.budget, decode_bs_divisor=a.divisor) \
            if mode == "pdmux" else None
        step = pm.step if pm is not None else eng.step
        g = torch.Generator().manual_seed(0)
        for _ in range(a.decode):
            eng.add_request(torch.randint(1, min(1000, cfg.vocab), (a.ctx,), generator=g).tolist(),
                            SamplingParams(max_new_tokens=2048, ignore_eos=True))
        for _ in range(10000):
            if not (eng.sched.waiting or eng.sched.prefilling or
                    (pm is not None and (pm.split is not None or pm.pending is not None))):
                break
            step()
        else:
            raise RuntimeError("decode requests were not all admitted")
        for _ in range(8):
            step()
        prompt = torch.randint(1, min(1000, cfg.vocab), (a.prompt,), generator=g).tolist()
        _window(step, eng, prompt)                     # warm-up window (graphs, lanes, allocator)
        res[mode] = _window(step, eng, prompt)
        if pm is not None:
            res["lanes_sms"] = pm.lanes.sms
            res["groups_used"] = sorted({g for g, _, _ in pm.log})
        del eng, pm
        torch.cuda.empty_cache()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
