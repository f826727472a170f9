"""HTTP front end: one engine loop thread per process, FastAPI routes.

    POST /generate     {"input_ids": [...], "max_new_tokens": n}  or {"prompts": [[...], ...], ...}
                       -> {"output_ids": [...]} / {"outputs": [[...], ...]}
                       "stream": true (one prompt) -> newline-delimited JSON as the tokens are produced:
                       {"token_ids": [...]} per engine step, then {"done": true, "output_ids": [...]}
                       "dp_rank": r pins the request to data-parallel rank r of a ranked deployment (a session's turns
                       stay on the rank that caches its prefix); default: the cache-aware balancer
    POST /flush_cache  drops cached prefixes (radix cache) once no request is running
    GET  /health       {"ok": true, "running": r, "waiting": w}
    GET  /metrics      Prometheus text: request / token / step counters, time to first token and per-request decode
                       rate quantiles (p50, p90, p99) over the finished requests

The SGLang endpoints the reference's gate drives (`tooling/serving-gate/cell_gate.py`: /generate, /flush_cache).
Token ids in, token ids out (the engine serves random-init models; tokenisation is the client's business).  One
engine per process.  `EngineLoop` serves a single-rank engine; `RankedEngineLoop` serves an engine spread over ranks
(one process per GPU, rank 0 holds the HTTP server): tensor-parallel ranks receive every request in the same order,
data-parallel ranks the requests the cache-aware balancer assigns them, and all ranks step in lockstep.
    POST /shutdown     stops the engine loop (every rank of a ranked deployment)"""
from __future__ import annotations

import threading
import time
from typing import Optional

from ..engine.engine import Engine
from ..engine.scheduler import SamplingParams


class EngineLoop:
    """Owns the engine; requests are queued from HTTP threads and stepped by one loop thread."""

    def __init__(self, engine: Engine, idle_sleep: float = 0.001):
        self.engine = engine
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)
        self.done: dict = {}
        self.counters = {"requests": 0, "tokens_out": 0, "steps": 0}
        self.t_submit: dict = {}                  # rid -> submit time; first-token time once known
        self.t_first: dict = {}
        self.ttft: list = []                      # seconds, finished requests
        self.user_rate: list = []                 # decode tok/s per finished request (after its first token)
        self.stream: dict = {}                    # rid -> tokens produced so far (streamed requests)
        self.meta: dict = {}                      # rid -> {"prompt_tokens", "cached_tokens"} of finished requests
        self.stop = False
        self.idle_sleep = idle_sleep
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def submit(self, prompt: list, max_new: int, stream: bool = False, dp_rank: Optional[int] = None) -> int:
        with self.lock:
            r = self.engine.add_request(list(prompt), SamplingParams(max_new_tokens=max_new))
            self.counters["requests"] += 1
            self.t_submit[r.rid] = time.perf_counter()
            if stream:
                self.stream[r.rid] = []
            self.cv.notify_all()
            return r.rid

    def _emit(self, rid, toks) -> None:
        """Tokens of one engine step for request rid (lock held)."""
        if rid in self.stream:
            self.stream[rid].extend(toks)

    def stream_tokens(self, rid: int, timeout: float = 600.0):
        """Generator of newline-delimited JSON for a streamed request: each batch of new tokens, then the final
        record (the request's output)."""
        import json
        sent, deadline = 0, time.time() + timeout
        while True:
            with self.lock:
                while True:
                    toks = self.stream.get(rid, [])
                    done = rid in self.done
                    if len(toks) > sent or done:
                        break
                    if time.time() > deadline:
                        raise TimeoutError(f"request {rid} not finished in {timeout} s")
                    self.cv.wait(1.0)
                new = toks[sent:]
                sent = len(toks)
                final = None
                if done:
                    final = self.done.pop(rid)
                    meta = self.meta.pop(rid, {})
                    self.stream.pop(rid, None)
            if new:
                yield json.dumps({"token_ids": new}) + "\n"
            if final is not None:
                yield json.dumps({"done": True, "output_ids": final, "meta_info": meta}) + "\n"
                return

    def wait(self, rid: int, timeout: float = 600.0) -> list:
        deadline = time.time() + timeout
        with self.lock:
            while rid not in self.done:
                left = deadline - time.time()
                if left <= 0:
                    raise TimeoutError(f"request {rid} not finished in {timeout} s")
                self.cv.wait(left)
            return self.done.pop(rid)

    def _run(self) -> None:
        while not self.stop:
            with self.lock:
                if not self.engine.has_work():
                    self.cv.wait(0.05)
                    continue
                out = self.engine.step()
                now = time.perf_counter()
                self.counters["steps"] += 1
                self.counters["tokens_out"] += sum(len(v) for v in out.values())
                for rid, toks in out.items():
                    self.t_first.setdefault(rid, now)
                    self._emit(rid, toks)
                for r in self.engine.finished:
                    if r.rid not in self.done:
                        self.done[r.rid] = list(r.output)
                        self.meta[r.rid] = {"prompt_tokens": r.prompt_len, "cached_tokens": r.cached_tokens}
                        self._record(r, now)
                self.engine.finished.clear()
                self.cv.notify_all()

    def _record(self, r, now: float) -> None:
        t0, t1 = self.t_submit.pop(r.rid, None), self.t_first.pop(r.rid, None)
        if t0 is None or t1 is None:
            return
        self.ttft.append(t1 - t0)
        if len(r.output) > 1 and now > t1:
            self.user_rate.append((len(r.output) - 1) / (now - t1))
        del self.ttft[:-10000], self.user_rate[:-10000]          # a sliding window of recent requests

    def quantiles(self) -> dict:
        """{"ttft_s": {q: v}, "user_tok_s": {q: v}} over the finished requests in the window (q = 0.5, 0.9, 0.99)."""
        def qs(v):
            if not v:
                return {}
            s = sorted(v)
            return {q: s[min(len(s) - 1, int(q * len(s)))] for q in (0.5, 0.9, 0.99)}
        return {"ttft_s": qs(self.ttft), "user_tok_s": qs(self.user_rate)}

    def shutdown(self) -> None:
        self.stop = True
        self.thread.join(timeout=5)


class RankedEngineLoop(EngineLoop):
    """The engine loop of a deployment over `world` ranks of a CPU process group `group` (gloo), one per process;
    rank 0's instance takes the HTTP requests.  Each pass: rank 0 broadcasts the requests that arrived since the last
    pass (and the stop flag); mode "tp": every rank adds every request, in order, so the ranks' schedulers stay
    identical; mode "dp": the cache-aware balancer (`engine/dp_policy.DPBalancer`, the same on every rank) assigns
    each request to one rank, the ranks all-gather their scheduler facts and take the joint decode-burst / prefill
    budget decisions (as `Engine.generate_dp`); every rank steps (idle ranks join the expert exchanges); outputs of
    finished requests are gathered to rank 0.  Rank 0 broadcasts at least every `heartbeat` seconds, so waiting
    ranks never reach the group's timeout while the server is idle."""

    def __init__(self, engine: Engine, rank: int, world: int, group, mode: str = "dp", heartbeat: float = 0.05):
        if mode not in ("dp", "tp"):
            raise ValueError(mode)
        self.rank, self.world, self.group, self.mode, self.heartbeat = rank, world, group, mode, heartbeat
        self.inbox: list = []                     # rank 0: (global id, prompt, max_new) since the last pass
        self.next_id = 0
        self.local_to_global: dict = {}
        self.delayed = 0
        if mode == "dp":
            from ..engine.dp_policy import DPBalancer
            self.balancer = DPBalancer(world)
        super().__init__(engine)

    def submit(self, prompt: list, max_new: int, stream: bool = False, dp_rank: Optional[int] = None) -> int:
        with self.lock:
            gid = self.next_id
            self.next_id += 1
            pin = None if dp_rank is None or self.mode != "dp" else int(dp_rank) % self.world
            self.inbox.append((gid, list(prompt), int(max_new), pin))
            self.counters["requests"] += 1
            self.t_submit[gid] = time.perf_counter()
            if stream:
                self.stream[gid] = []
            self.cv.notify_all()
            return gid

    def _run(self) -> None:
        import torch
        import torch.distributed as dist
        from ..engine.burst import RankFacts, dp_hold
        from ..engine.dp_policy import prefill_budget
        eng = self.engine
        any_work = False                            # some rank had work at the last pass (the gathered flag)
        while True:
            with self.lock:
                if self.rank == 0 and not self.inbox and not self.stop and not eng.has_work() and not any_work:
                    self.cv.wait(self.heartbeat)
                msg = [(list(self.inbox), self.stop)] if self.rank == 0 else [None]
                self.inbox.clear()
            dist.broadcast_object_list(msg, src=0, group=self.group)
            new, stop = msg[0]
            if stop:
                return
            with self.lock:
                for gid, prompt, max_new, pin in new:
                    if self.mode == "dp" and pin is not None:
                        self.balancer.pin(prompt, pin, t=float(gid))
                        mine = pin == self.rank
                    else:
                        mine = self.mode == "tp" or self.balancer.route(prompt, t=float(gid)) == self.rank
                    if mine:
                        r = eng.add_request(prompt, SamplingParams(max_new_tokens=max_new))
                        self.local_to_global[r.rid] = gid
                hold, cap, work = None, 0, eng.has_work()
                if self.mode == "dp":
                    f = eng.sched.facts()
                    row = torch.tensor(f[:5] + [self.delayed, f[5], int(work)], dtype=torch.int64)
                    parts = [torch.empty_like(row) for _ in range(self.world)]
                    dist.all_gather(parts, row, group=self.group)
                    rows = [p.tolist() for p in parts]
                    work = any(r[7] for r in rows)
                    if work:
                        hold = dp_hold([RankFacts.from_row(r[:6]) for r in rows], eng.ecfg.decode_burst,
                                       eng.ecfg.burst_queue_cap, eng.ecfg.max_delay_passes)
                        cap = prefill_budget([r[6] for r in rows], eng.ecfg.chunked_prefill,
                                             min_tokens=min(2048, eng.ecfg.chunked_prefill), page=eng.ecfg.page_size)
                any_work = work
                finished, emitted = [], []
                if work:
                    out = eng.step(hold=hold, chunk_cap=cap)
                    self.delayed = self.delayed + 1 if hold else 0
                    now = time.perf_counter()
                    self.counters["steps"] += 1
                    self.counters["tokens_out"] += sum(len(v) for v in out.values())
                    for rid, toks in out.items():
                        gid = self.local_to_global.get(rid)
                        if gid is not None:
                            self.t_first.setdefault(gid, now)
                            emitted.append((gid, list(toks)))
                    for r in eng.finished:
                        gid = self.local_to_global.pop(r.rid, None)
                        if gid is not None:
                            finished.append((gid, list(r.output), len(r.output), r.prompt_len, r.cached_tokens))
                    eng.finished.clear()
            if self.mode == "dp":                 # every rank's new tokens and finished requests reach rank 0
                got = [None] * self.world if self.rank == 0 else None
                dist.gather_object((emitted, finished), got, dst=0, group=self.group)
                if self.rank == 0:
                    emitted = [x for part in got for x in part[0]]
                    finished = [x for part in got for x in part[1]]
                else:
                    emitted, finished = [], []
            if self.rank == 0 and emitted:
                with self.lock:
                    now = time.perf_counter()
                    for gid, toks in emitted:
                        self.t_first.setdefault(gid, now)
                        self._emit(gid, toks)
                    self.cv.notify_all()
            if self.rank == 0 and finished:
                with self.lock:
                    now = time.perf_counter()
                    for gid, output, n, plen, cached in finished:
                        self.done[gid] = output
                        self.meta[gid] = {"prompt_tokens": plen, "cached_tokens": cached}
                        t0, t1 = self.t_submit.pop(gid, None), self.t_first.pop(gid, None)
                        if t0 is not None:
                            self.ttft.append((t1 or now) - t0)
                            if t1 is not None and n > 1 and now > t1:
                                self.user_rate.append((n - 1) / (now - t1))
                    self.cv.notify_all()

    def shutdown(self) -> None:
        with self.lock:
            self.stop = True
            self.cv.notify_all()
        self.thread.join(timeout=30)


def make_app(loop: EngineLoop):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse

    app = FastAPI()

    @app.post("/generate")
    def generate(body: dict):
        max_new = int(body.get("max_new_tokens", body.get("sampling_params", {}).get("max_new_tokens", 16)))
        pin = body.get("dp_rank")
        if "prompts" in body:
            rids = [loop.submit(p, max_new, dp_rank=pin) for p in body["prompts"]]
            outs = [loop.wait(r) for r in rids]
            with loop.lock:
                for r in rids:
                    loop.meta.pop(r, None)
            return {"outputs": outs}
        if "input_ids" not in body:
            raise HTTPException(400, "input_ids or prompts required")
        if body.get("stream"):
            rid = loop.submit(body["input_ids"], max_new, stream=True, dp_rank=pin)
            return StreamingResponse(loop.stream_tokens(rid), media_type="application/x-ndjson")
        rid = loop.submit(body["input_ids"], max_new, dp_rank=pin)
        out = loop.wait(rid)
        with loop.lock:
            meta = loop.meta.pop(rid, {})
        return {"output_ids": out, "meta_info": meta}

    @app.post("/flush_cache")
    def flush_cache():
        with loop.lock:
            if loop.engine.sched.running:
                return {"flushed": False, "reason": "requests running"}
            cache = getattr(loop.engine.runner, "prefix_cache", None)
            if cache is not None:
                cache.clear()
            return {"flushed": True}

    @app.post("/shutdown")
    def shutdown():
        threading.Thread(target=loop.shutdown, daemon=True).start()
        return {"stopping": True}

    @app.get("/health")
    def health():
        s = loop.engine.sched
        return {"ok": True, "running": len(s.running), "waiting": len(s.waiting)}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        with loop.lock:
            c = dict(loop.counters)
            qs = loop.quantiles()
        lines = [f"iob_{k}_total {v}\n" for k, v in c.items()]
        for name, vals in qs.items():
            lines += [f'iob_{name}{{quantile="{q}"}} {v:.6g}\n' for q, v in vals.items()]
        return "".join(lines)

    return app


def serve(engine: Engine, host: str = "127.0.0.1", port: int = 30000, block: bool = True, loop=None):
    """Run the server (uvicorn) over `loop` (default: a single-rank EngineLoop).  block=False returns (server, thread,
    loop) for tests / embedding."""
    import uvicorn
    loop = loop or EngineLoop(engine)
    config = uvicorn.Config(make_app(loop), host=host, port=port, log_level="warning")
    server = uvicorn.Server(config)
    if block:
        server.run()
        return None
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.02)
    return server, th, loop


def main(argv: Optional[list] = None) -> None:
    from ..config import model_config, resolve
    import argparse
    p = argparse.ArgumentParser(add_help=False)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=30000)
    p.add_argument("--max-seq", type=int, default=8192)
    ns, rest = p.parse_known_args(argv)
    ecfg = resolve(rest)
    import os
    if int(os.environ.get("WORLD_SIZE", "1")) == 1:
        serve(Engine(ecfg, model_config(ecfg.model), max_seq=ns.max_seq), ns.host, ns.port)
        return
    # one process per GPU (torchrun): rank 0 serves HTTP; tp > 1 -> every rank gets every request, else DP ranks
    import torch
    import torch.distributed as dist
    from ..parallel import dist as D
    info = D.init("nccl")
    ecfg.device = f"cuda:{info.local_rank}"
    world = dist.group.WORLD
    if ecfg.tp > 1:
        eng = Engine(ecfg, model_config(ecfg.model), max_seq=ns.max_seq, tp_rank=info.rank, tp=ecfg.tp,
                     all_reduce=D.nccl_all_reduce, argmax_merge=D.argmax_merge)
        mode = "tp"
    else:
        eng = Engine(ecfg, model_config(ecfg.model), max_seq=ns.max_seq, ep_rank=info.rank,
                     ep_group=world if ecfg.ep > 1 else None, dcp_rank=info.rank,
                     dcp_group=world if ecfg.dcp > 1 else None)
        mode = "tp" if ecfg.dcp > 1 else "dp"      # context-parallel ranks run the same requests
    loop = RankedEngineLoop(eng, info.rank, info.world, info.cpu_group, mode)
    if info.rank == 0:
        serve(eng, ns.host, ns.port, loop=loop)
    else:
        loop.thread.join()
    torch.cuda.synchronize()
    D.shutdown()


if __name__ == "__main__":
    main()
