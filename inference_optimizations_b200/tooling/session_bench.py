"""Session load generator for the HTTP front end (`server/http.py`): N concurrent users, each with its own context,
several turns -- the workload the reference's serving gate drives (`tooling/serving-gate/dc_bench.py:1-20`).

Protocol per session (all sessions run at once):
  turn 1: prompt = a unique random prefix of `prefix` tokens, generate `output` tokens      [cold: full prefill]
  turn t: prompt = the previous prompt + its output + `question` new tokens, generate `output` [warm: prefix cached]
Each turn is one streamed `/generate` (token ids in, newline-delimited JSON out), so the time to the first token is
measured at the client.  With `dp` > 1 the turns of session s go to data-parallel rank s % dp (`dp_rank`), the rank
that holds the session's prefix.

Summary (`summarize`, pure, so it is tested without a server): over the warm turns, aggregate output tok/s across the
warm window, per-user decode tok/s p50 / p99 ((output tokens - 1) / (turn wall - TTFT); p99 is the slow tail, the
1st percentile of the rates), TTFT p50 / p90 / p99 / max, turn wall p50 / p99, prefix hit rate (cached prompt tokens
/ prompt tokens, from the server's meta_info); over the cold turns, prefill tok/s and TTFT.

    python -m inference_optimizations_b200.tooling.session_bench --url http://127.0.0.1:30000 \
        --sessions 64 --turns 4 --prefix 8192 --question 128 --output 256 --vocab 129280
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from dataclasses import asdict, dataclass
from typing import Optional


@dataclass
class SessionSpec:
    sessions: int = 8
    turns: int = 3
    prefix: int = 512
    question: int = 32
    output: int = 32
    vocab: int = 32000
    dp: int = 0                 # > 1: pin session s to data-parallel rank s % dp
    seed: int = 0
    timeout_s: float = 600.0


@dataclass
class TurnResult:
    session: int
    turn: int
    prompt_tokens: int
    cached_tokens: int
    completion_tokens: int
    ttft_s: float
    wall_s: float
    t_start: float
    error: Optional[str] = None
    tokens: Optional[list] = None          # the turn's output ids (not part of the summary)

    @property
    def t_end(self) -> float:
        return self.t_start + self.wall_s

    @property
    def decode_tok_s(self) -> Optional[float]:
        d = self.wall_s - self.ttft_s
        return (self.completion_tokens - 1) / d if self.completion_tokens > 1 and d > 0 else None


def _pct(xs: list, q: float) -> Optional[float]:
    """Nearest-rank percentile (q in [0, 1]) of xs; None when empty."""
    if not xs:
        return None
    s = sorted(xs)
    return s[min(len(s) - 1, max(0, int(round(q * (len(s) - 1)))))]


def _r(x: Optional[float], nd: int = 3) -> Optional[float]:
    return None if x is None else round(x, nd)


def summarize(results: list, spec: SessionSpec) -> dict:
    ok = [r for r in results if r.error is None]
    bad = [r for r in results if r.error is not None]
    warm = [r for r in ok if r.turn >= 2]
    cold = [r for r in ok if r.turn == 1]

    def window_rate(rows):
        if not rows:
            return None
        t0, t1 = min(r.t_start for r in rows), max(r.t_end for r in rows)
        return sum(r.completion_tokens for r in rows) / (t1 - t0) if t1 > t0 else None

    def hit(rows):
        p = sum(r.prompt_tokens for r in rows)
        return sum(r.cached_tokens for r in rows) / p if p else None

    rates = [r.decode_tok_s for r in warm if r.decode_tok_s is not None]
    ttft = [r.ttft_s for r in warm]
    walls = [r.wall_s for r in warm]
    prefill = None
    if cold:
        t0, t1 = min(r.t_start for r in cold), max(r.t_start + r.ttft_s for r in cold)
        new = sum(r.prompt_tokens - r.cached_tokens for r in cold)
        prefill = new / (t1 - t0) if t1 > t0 else None
    return {
        "spec": asdict(spec),
        "sessions_completed": len({r.session for r in ok if r.turn == spec.turns}),
        "requests_ok": len(ok), "requests_failed": len(bad),
        "error_sample": sorted({(r.error or "")[:160] for r in bad})[:3],
        "warm": {"agg_out_tok_s": _r(window_rate(warm)),
                 "per_user_tok_s": {"p50": _r(_pct(rates, 0.5)), "p99": _r(_pct(rates, 0.01))},
                 "ttft_s": {"p50": _r(_pct(ttft, 0.5), 4), "p90": _r(_pct(ttft, 0.9), 4),
                            "p99": _r(_pct(ttft, 0.99), 4), "max": _r(max(ttft) if ttft else None, 4)},
                 "turn_wall_s": {"p50": _r(_pct(walls, 0.5), 4), "p99": _r(_pct(walls, 0.99), 4)},
                 "hit_rate": _r(hit(warm), 4),
                 "prompt_tokens_mean": _r(sum(r.prompt_tokens for r in warm) / len(warm), 1) if warm else None,
                 "out_tokens_mean": _r(sum(r.completion_tokens for r in warm) / len(warm), 1) if warm else None},
        "cold": {"prefill_tok_s": _r(prefill), "ttft_s": {"p50": _r(_pct([r.ttft_s for r in cold], 0.5), 4),
                                                          "p99": _r(_pct([r.ttft_s for r in cold], 0.99), 4)},
                 "hit_rate": _r(hit(cold), 4)},
        "all": {"agg_out_tok_s": _r(window_rate(ok))},
    }


async def _turn(http, url: str, s: int, turn: int, prompt: list, spec: SessionSpec) -> tuple:
    body = {"input_ids": prompt, "max_new_tokens": spec.output, "stream": True}
    if spec.dp > 1:
        body["dp_rank"] = s % spec.dp
    t0 = time.perf_counter()
    ttft, toks, meta = None, [], {}
    async with http.post(url + "/generate", json=body) as resp:
        if resp.status != 200:
            raise RuntimeError(f"HTTP {resp.status}: {(await resp.text())[:200]}")
        async for line in resp.content:
            line = line.strip()
            if not line:
                continue
            msg = json.loads(line)
            if msg.get("token_ids"):
                if ttft is None:
                    ttft = time.perf_counter() - t0
                toks.extend(msg["token_ids"])
            if msg.get("done"):
                toks = msg.get("output_ids", toks)
                meta = msg.get("meta_info", {})
    wall = time.perf_counter() - t0
    return TurnResult(s, turn, len(prompt), int(meta.get("cached_tokens", 0)), len(toks),
                      ttft if ttft is not None else wall, wall, t0, tokens=list(toks)), toks


async def _session(http, url: str, s: int, spec: SessionSpec) -> list:
    rng = random.Random(spec.seed * 1_000_003 + s)
    prompt = [rng.randrange(1, spec.vocab) for _ in range(spec.prefix)]
    out = []
    for turn in range(1, spec.turns + 1):
        try:
            res, toks = await _turn(http, url, s, turn, prompt, spec)
        except Exception as e:                       # noqa: BLE001 -- one failed turn ends the session, recorded
            out.append(TurnResult(s, turn, len(prompt), 0, 0, 0.0, 0.0, time.perf_counter(), error=repr(e)))
            break
        out.append(res)
        prompt = prompt + toks + [rng.randrange(1, spec.vocab) for _ in range(spec.question)]
    return out


async def run(url: str, spec: SessionSpec) -> list:
    import aiohttp
    timeout = aiohttp.ClientTimeout(total=spec.timeout_s)
    conn = aiohttp.TCPConnector(limit=0)
    async with aiohttp.ClientSession(timeout=timeout, connector=conn) as http:
        parts = await asyncio.gather(*[_session(http, url.rstrip("/"), s, spec) for s in range(spec.sessions)])
    return [r for p in parts for r in p]


def bench(url: str, spec: SessionSpec) -> dict:
    """Run the sessions against a live server and summarize."""
    return summarize(asyncio.run(run(url, spec)), spec)


def main(argv: Optional[list] = None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--url", default="http://127.0.0.1:30000")
    for f in ("sessions", "turns", "prefix", "question", "output", "vocab", "dp", "seed"):
        p.add_argument("--" + f, type=int, default=getattr(SessionSpec, f))
    p.add_argument("--timeout", type=float, default=600.0)
    a = p.parse_args(argv)
    spec = SessionSpec(a.sessions, a.turns, a.prefix, a.question, a.output, a.vocab, a.dp, a.seed, a.timeout)
    print(json.dumps(bench(a.url, spec)))


if __name__ == "__main__":
    main()
