"""A/B serving gate: one control arm and one arm with a single delta, the same synthetic sessions, warm-up, timed
rounds, several repeats with alternating arm order, and one JSON evidence record per arm -- the method of the
reference's cell gate (`tooling/serving-gate/cell_gate.py`; evidence schema `evidence/README.md`, methodology
`docs/methodology.md:13-34`: served throughput is compared arm against arm on the same box, never against a
number from another machine).

    python -m inference_optimizations_b200.tooling.serving_gate --model tiny_gqa --device cpu \
        --delta '{"decode_burst": 4}' --sessions 4 --prompt 96 --steps 8 --repeats 2 --out evidence.json

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
    a = ap.parse_args(argv)
    ecfg = EngineConfig(model=a.model, device=a.device, kv_dtype=a.kv, max_running=a.sessions,
                        cuda_graphs=a.device.startswith("cuda"))
    res = gate(ecfg, model_config(a.model), json.loads(a.delta), a.sessions, a.prompt, a.steps, a.warmup, a.repeats)
    s = json.dumps(res, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(s)
    print(json.dumps({"ratio": res["ratio"], "verdict": res["verdict"], "control_spread": res["control_spread"]}))


if __name__ == "__main__":
    main()
