"""Accuracy gate: teacher-forced comparison of a quantized-KV engine against a reference engine (the reference's
`tooling/accuracy-gate/accuracy_gate.py:456-594` method: per-position KL of next-token distributions, top-1
agreement, p99 |delta logprob| of the reference's own token, over many prompts; thresholds from a noise floor).

    python -m inference_optimizations_b200.tooling.accuracy_gate --model tiny_gqa --test-kv nvfp4 --ref-kv bf16

Both engines hold the same random-init weights (same seed); each prompt is scored in one teacher-forced pass per
engine (`runner.score`), so the comparison isolates the KV format.  The BASELINE target is KL <= 0.03 vs bf16 KV.
"""
from __future__ import annotations

import argparse
import json
from dataclasses import dataclass

import torch


@dataclass
class GateResult:
    kl_mean: float
    kl_p99: float
    top1: float
    dlogp_p99: float
    positions: int
    prompts: int

    def passed(self, kl_max: float = 0.03, top1_min: float = 0.0) -> bool:
        return self.kl_mean <= kl_max and self.top1 >= top1_min


def compare_logits(ref: torch.Tensor, test: torch.Tensor, temperature: float = 1.0) -> dict:
    """ref / test [T, V] logits -> per-position KL(ref || test), top-1 match, |delta logprob| of ref's argmax."""
    lr = torch.log_softmax(ref.float() / temperature, -1)
    lt = torch.log_softmax(test.float() / temperature, -1)
    kl = (lr.exp() * (lr - lt)).sum(-1)
    a = lr.argmax(-1)
    return {"kl": kl, "top1": (a == lt.argmax(-1)).float(),
            "dlogp": (lr.gather(1, a[:, None]) - lt.gather(1, a[:, None])).abs()[:, 0]}


def run_gate(ref_engine, test_engine, prompts: list, skip: int = 1) -> GateResult:
    kls, t1, dl = [], [], []
    for p in prompts:
        c = compare_logits(ref_engine.runner.score(p)[skip:], test_engine.runner.score(p)[skip:])
        kls.append(c["kl"])
        t1.append(c["top1"])
        dl.append(c["dlogp"])
    kl, top1, dlp = torch.cat(kls), torch.cat(t1), torch.cat(dl)
    return GateResult(kl.mean().item(), kl.quantile(0.99).item(), top1.mean().item(), dlp.quantile(0.99).item(),
                      kl.numel(), len(prompts))


def main(argv=None) -> None:
    from ..config import EngineConfig, model_config
    from ..engine.engine import Engine
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny_gqa")
    ap.add_argument("--test-kv", default="nvfp4")
    ap.add_argument("--ref-kv", default="bf16")
    ap.add_argument("--prompts", type=int, default=16)
    ap.add_argument("--len", type=int, default=256)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--kl-max", type=float, default=0.03)
    ap.add_argument("--layers", type=int, default=0, help="truncate the model to its first N layers (0 = all)")
    ap.add_argument("--first-dense", type=int, default=-1, help="MLA family: dense layers before the MoE layers")
    a = ap.parse_args(argv)
    cfg = model_config(a.model)
    from dataclasses import replace
    if a.layers:
        cfg = replace(cfg, num_layers=a.layers)
    if a.first_dense >= 0:
        cfg = replace(cfg, first_dense=a.first_dense)
    mk = lambda kv: Engine(EngineConfig(model=a.model, device=a.device, kv_dtype=kv, max_running=2,  # noqa: E731
                                        chunked_prefill=a.len, cuda_graphs=False), cfg, max_seq=a.len + 64)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab, (a.len,), generator=g).tolist() for _ in range(a.prompts)]
    res = run_gate(mk(a.ref_kv), mk(a.test_kv), prompts)
    print(json.dumps({"model": a.model, "layers": cfg.num_layers, "prompt_len": a.len, "ref_kv": a.ref_kv,
                      "test_kv": a.test_kv, **vars(res), "pass": res.passed(a.kl_max)}))


if __name__ == "__main__":
    main()
