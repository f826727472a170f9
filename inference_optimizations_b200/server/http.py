"""HTTP front end: one engine loop thread per process, FastAPI routes.

    POST /generate     {"input_ids": [...], "max_new_tokens": n}  or {"prompts": [[...], ...], ...}
                       -> {"output_ids": [...]} / {"outputs": [[...], ...]}
    POST /flush_cache  drops cached prefixes (radix cache) once no request is running
    GET  /health       {"ok": true, "running": r, "waiting": w}
    GET  /metrics      Prometheus text: requests, tokens, step counts

The SGLang endpoints the reference's gate drives (`tooling/serving-gate/cell_gate.py`: /generate, /flush_cache).
Token ids in, token ids out (the engine serves random-init models; tokenisation is the client's business).  One
engine per process: this front end serves a single-rank engine; a tensor-parallel deployment must feed every rank's
engine the same requests in the same order (`engine/engine.py`), which this module does not do."""
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
        self.stop = False
        self.idle_sleep = idle_sleep
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def submit(self, prompt: list, max_new: int) -> int:
        with self.lock:
            r = self.engine.add_request(list(prompt), SamplingParams(max_new_tokens=max_new))
            self.counters["requests"] += 1
            self.cv.notify_all()
            return r.rid

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
                self.counters["steps"] += 1
                self.counters["tokens_out"] += sum(len(v) for v in out.values())
                for r in self.engine.finished:
                    if r.rid not in self.done:
                        self.done[r.rid] = list(r.output)
                self.engine.finished.clear()
                self.cv.notify_all()

    def shutdown(self) -> None:
        self.stop = True
        self.thread.join(timeout=5)


def make_app(loop: EngineLoop):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse

    app = FastAPI()

    @app.post("/generate")
    def generate(body: dict):
        max_new = int(body.get("max_new_tokens", body.get("sampling_params", {}).get("max_new_tokens", 16)))
        if "prompts" in body:
            rids = [loop.submit(p, max_new) for p in body["prompts"]]
            return {"outputs": [loop.wait(r) for r in rids]}
        if "input_ids" not in body:
            raise HTTPException(400, "input_ids or prompts required")
        return {"output_ids": loop.wait(loop.submit(body["input_ids"], max_new))}

    @app.post("/flush_cache")
    def flush_cache():
        with loop.lock:
            if loop.engine.sched.running:
                return {"flushed": False, "reason": "requests running"}
            cache = getattr(loop.engine.runner, "prefix_cache", None)
            if cache is not None:
                cache.clear()
            return {"flushed": True}

    @app.get("/health")
    def health():
        s = loop.engine.sched
        return {"ok": True, "running": len(s.running), "waiting": len(s.waiting)}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        c = loop.counters
        return "".join(f"iob_{k}_total {v}\n" for k, v in c.items())

    return app


def serve(engine: Engine, host: str = "127.0.0.1", port: int = 30000, block: bool = True):
    """Run the server (uvicorn).  block=False returns (server, thread, loop) for tests / embedding."""
    import uvicorn
    loop = EngineLoop(engine)
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
    serve(Engine(ecfg, model_config(ecfg.model), max_seq=ns.max_seq), ns.host, ns.port)


if __name__ == "__main__":
    main()
