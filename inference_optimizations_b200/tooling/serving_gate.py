"""A/B serving gate: one control arm and one arm with a single delta, the same synthetic sessions, warm-up, timed
rounds, several repeats with alternating arm order, and one JSON evidence record per arm -- the method of the
reference's cell gate (`tooling/serving-gate/cell_gate.py`; evidence schema `evidence/README.md`, methodology
`docs/methodology.md:13-34`: served throughput is compared arm against arm on the same box, never against a
number from another machine).

    python -m inference_optimizations_b200.tooling.serving_gate --model tiny_gqa --device cpu \
        --delta '{"decode_burst": 4}' --sessions 4 --prompt 96 --steps 8 --repeats 2 --out evidence.json
    # the same gate through the HTTP front end, multi-turn sessions from the session load generator:
    python -m inference_optimizations_b200.tooling.serving_gate --http --model tiny_gqa --device cpu \
        --delta '{"decode_burst": 4}' --sessions 4 --prompt 96 --turns 3 --repeats 2

Each run builds a fresh engine for the arm, registers `sessions` requests with `prompt` random tokens, prefills them
(untimed), runs `warmup` engine steps, then times `steps` steps (CUDA events on a GPU, wall clock on the CPU) and
records aggregate output tok/s and per-user tok/s.  The verdict compares the arm means against the control's
repeat-to-repeat spread (a delta inside the noise is reported as neutral).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import time
from dataclasses import asdict, replace
from typing import Optional

import torch


def _digest(d: dict) -> str:
    return hashlib.sha256(json.dumps(d, sort_keys=True, default=str).encode()).hexdigest()[:16]


def run_arm(ecfg, mcfg, sessions: int, prompt: int, steps: int, warmup: int, seed: int) -> dict:
    from ..engine.engine import Engine
    from ..engine.scheduler import SamplingParams
    eng = Engine(ecfg, mcfg, max_seq=prompt + warmup * 4 + steps * 4 + 64)
    g = torch.Generator().manual_seed(seed)
    reqs = [eng.add_request(torch.randint(1, mcfg.vocab, (prompt,), generator=g).tolist(),
                            SamplingParams(max_new_tokens=warmup * 4 + steps * 4 + 32)) for _ in range(sessions)]
    while any(r.prefilled < r.prompt_len for r in reqs):          # prefill (untimed)
        eng.step()
    for _ in range(warmup):
        eng.step()
    cuda = str(ecfg.device).startswith("cuda")
    if cuda:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    t0 = time.perf_counter()
    toks = 0
    for _ in range(steps):
        out = eng.step()
        toks += sum(len(v) for v in out.values())
    if cuda:
        e1.record()
        torch.cuda.synchronize()
        secs = e0.elapsed_time(e1) / 1e3
    else:
        secs = time.perf_counter() - t0
    agg = toks / max(secs, 1e-9)
    return {"sessions": sessions, "warm_agg_out_tok_s": round(agg, 3), "warm_per_user_tok_s": round(agg / sessions, 3),
            "steps": steps, "seconds": round(secs, 6), "tokens": toks}


def gate(ecfg, mcfg, delta: dict, sessions: int = 4, prompt: int = 96, steps: int = 8, warmup: int = 2,
         repeats: int = 2, seed: int = 0, cell: str = "local") -> dict:
    """Run control and treatment `repeats` times each, alternating which goes first."""
    arms = {"control": ecfg, "delta": replace(ecfg, **delta)}
    runs = {"control": [], "delta": []}
    for rep in range(repeats):
        order = ("control", "delta") if rep % 2 == 0 else ("delta", "control")
        for name in order:
            runs[name].append(run_arm(arms[name], mcfg, sessions, prompt, steps, warmup, seed + rep))
    started = time.strftime("%Y-%m-%dT%H:%M:%S")
    rec = {}
    for name, cfg in arms.items():
        vals = [r["warm_agg_out_tok_s"] for r in runs[name]]
        rec[name] = {"cell": cell, "arm": name, "delta": delta if name == "delta" else {},
                     "config_digest": _digest(asdict(cfg)), "model": getattr(mcfg, "name", "?"),
                     "repeats": repeats, "started": started, "runs": runs[name],
                     "mean_agg_out_tok_s": round(sum(vals) / len(vals), 3)}
    c = [r["warm_agg_out_tok_s"] for r in runs["control"]]
    spread = (max(c) - min(c)) / max(1e-9, sum(c) / len(c))
    ratio = rec["delta"]["mean_agg_out_tok_s"] / max(1e-9, rec["control"]["mean_agg_out_tok_s"])
    verdict = "neutral" if abs(ratio - 1.0) <= spread else ("better" if ratio > 1.0 else "worse")
    return {"arms": rec, "ratio": round(ratio, 4), "control_spread": round(spread, 4), "verdict": verdict}


def _verdict(runs: dict, key) -> tuple:
    c = [key(r) for r in runs["control"]]
    d = [key(r) for r in runs["delta"]]
    mc, md = sum(c) / len(c), sum(d) / len(d)
    spread = (max(c) - min(c)) / max(1e-9, mc)
    ratio = md / max(1e-9, mc)
    verdict = "neutral" if abs(ratio - 1.0) <= spread else ("better" if ratio > 1.0 else "worse")
    return ratio, spread, verdict


def launch_server(flags: list, port: int, max_seq: int = 8192, gpus: int = 1, timeout_s: float = 600.0):
    """Start `server/http.py` in a child process (torchrun over `gpus` ranks when > 1) with engine flags `flags`
    (EngineConfig CLI), wait for /health -> (url, stop): stop() posts /shutdown and reaps the process group."""
    import os
    import signal
    import subprocess
    import sys
    import urllib.request
    mod = ["-m", "inference_optimizations_b200.server.http", "--port", str(port), "--max-seq", str(max_seq)] + flags
    if gpus > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
               "--master-addr", "127.0.0.1", "--master-port", str(port + 1)] + mod
    else:
        cmd = [sys.executable] + mod
    proc = subprocess.Popen(cmd, start_new_session=True)
    url = f"http://127.0.0.1:{port}"
    deadline = time.time() + timeout_s
    while True:
        if proc.poll() is not None:
            raise RuntimeError(f"server exited with {proc.returncode} before answering /health")
        try:
            with urllib.request.urlopen(url + "/health", timeout=2) as r:
                if r.status == 200:
                    break
        except OSError:
            pass
        if time.time() > deadline:
            os.killpg(proc.pid, signal.SIGTERM)
            raise TimeoutError("server did not answer /health")
        time.sleep(0.5)

    def stop():
        try:
            urllib.request.urlopen(urllib.request.Request(url + "/shutdown", method="POST"), timeout=10)
        except OSError:
            pass
        try:
            proc.wait(timeout=60)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGTERM)
            proc.wait(timeout=30)

    return url, stop


def gate_http(launchers: dict, spec, repeats: int = 2, cell: str = "local", delta: Optional[dict] = None) -> dict:
    """The A/B gate through the HTTP front end: for each repeat (arm order alternating) launch the arm's server
    (`launchers[name]() -> (url, stop)`, "control" and "delta"), drive it with the session load generator
    (`tooling/session_bench.py`: concurrent multi-turn users, streamed turns, DP-rank pinning), tear it down, and
    compare the arms on warm aggregate output tok/s against the control's repeat-to-repeat spread.  Evidence: one
    record per arm with every run's session summary."""
    from .session_bench import bench
    runs = {"control": [], "delta": []}
    for rep in range(repeats):
        for name in (("control", "delta") if rep % 2 == 0 else ("delta", "control")):
            url, stop = launchers[name]()
            try:
                runs[name].append(bench(url, spec))
            finally:
                stop()
    key = lambda r: r["warm"]["agg_out_tok_s"] or 0.0  # noqa: E731
    ratio, spread, verdict = _verdict(runs, key)
    started = time.strftime("%Y-%m-%dT%H:%M:%S")
    rec = {name: {"cell": cell, "arm": name, "delta": (delta or {}) if name == "delta" else {}, "repeats": repeats,
                  "started": started, "sessions_spec": runs[name][0]["spec"] if runs[name] else None,
                  "runs": runs[name], "mean_warm_agg_out_tok_s": round(sum(map(key, runs[name])) / len(runs[name]), 3)}
           for name in runs}
    return {"arms": rec, "ratio": round(ratio, 4), "control_spread": round(spread, 4), "verdict": verdict}


def main(argv: Optional[list] = None) -> None:
    from ..config import EngineConfig, model_config
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny_gqa")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--kv", default="nvfp4")
    ap.add_argument("--delta", required=True, help="JSON dict of EngineConfig fields the treatment arm changes")
    ap.add_argument("--sessions", type=int, default=4)
    ap.add_argument("--prompt", type=int, default=96)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--repeats", type=int, default=2)
    ap.add_argument("--out", default="")
    ap.add_argument("--http", action="store_true",
                    help="serve each arm over HTTP (server/http.py) and drive it with the session load generator")
    ap.add_argument("--gpus", type=int, default=1, help="--http: ranks per server (torchrun)")
    ap.add_argument("--port", type=int, default=30100)
    ap.add_argument("--turns", type=int, default=3)
    ap.add_argument("--question", type=int, default=32)
    ap.add_argument("--output", type=int, default=32)
    ap.add_argument("--dp", type=int, default=0, help="--http: pin session s to data-parallel rank s % dp")
    a = ap.parse_args(argv)
    delta = json.loads(a.delta)
    if a.http:
        from .session_bench import SessionSpec
        mcfg = model_config(a.model)
        base = ["--model", a.model, "--device", a.device, "--kv-dtype", a.kv, "--max-running", str(a.sessions)]
        flags = {"control": base,
                 "delta": base + [x for k, v in delta.items() for x in ("--" + k.replace("_", "-"), str(v))]}
        spec = SessionSpec(a.sessions, a.turns, a.prompt, a.question, a.output, mcfg.vocab, a.dp)
        max_seq = a.prompt + a.turns * (a.question + a.output) + 128
        launchers = {n: (lambda f=f: launch_server(f, a.port, max_seq, a.gpus)) for n, f in flags.items()}
        res = gate_http(launchers, spec, a.repeats, delta=delta)
    else:
        ecfg = EngineConfig(model=a.model, device=a.device, kv_dtype=a.kv, max_running=a.sessions,
                            cuda_graphs=a.device.startswith("cuda"))
        res = gate(ecfg, model_config(a.model), delta, a.sessions, a.prompt, a.steps, a.warmup, a.repeats)
    s = json.dumps(res, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(s)
    print(json.dumps({"ratio": res["ratio"], "verdict": res["verdict"], "control_spread": res["control_spread"]}))


if __name__ == "__main__":
    main()
