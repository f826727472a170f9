"""Accuracy gate statistics on CPU: the one-sided exact McNemar p-value against scipy's binomial test, paired
exact-match counting, noise-widened thresholds and the verdict logic, and one small end-to-end gate (bf16 vs FP8 KV,
with calibration and oracle exact-match items) on the tiny model."""
import pytest
from scipy.stats import binomtest

from inference_optimizations_b200.tooling import accuracy_gate as G


@pytest.mark.parametrize("b,c", [(0, 0), (3, 0), (5, 1), (10, 4), (4, 10), (30, 12), (1, 1)])
def test_mcnemar_matches_binomial_tail(b, c):
    want = 1.0 if b + c == 0 else binomtest(b, b + c, 0.5, alternative="greater").pvalue
    assert G.mcnemar_one_sided(b, c) == pytest.approx(want, rel=1e-12)


def test_exact_match_pairs():
    ans = [[1, 2], [3], [4, 4], [5]]
    ctl = [[1, 2, 9], [3, 0], [4, 0], [0]]         # right, right, wrong, wrong
    arm = [[1, 2], [0], [4, 4, 4], [0]]            # right, wrong, right, wrong
    em = G.exact_match(ctl, arm, ans)
    assert (em.control_correct, em.arm_correct, em.only_control, em.only_arm) == (2, 2, 1, 1)
    assert em.drop_pts == 0.0 and em.p_arm_worse == pytest.approx(0.75)


def test_thresholds_widen_with_noise_and_verdict():
    noise = {"kl_mean": 0.01, "kl_p99": 0.01, "top1": 0.995, "dlogp_p99": 0.01, "em_discordant_pts": 1.0}
    th = G.effective_thresholds(noise)
    assert th["kl_mean_max"] == pytest.approx(0.03) and th["top1_agree_min"] == pytest.approx(0.97)
    assert th["em_drop_max_pts"] == pytest.approx(3.0)
    good = G.GateResult(0.02, 0.2, 0.98, 0.3, 1000, 200)
    assert G.verdict(good, None, noise)["pass"] and not G.verdict(good, None, None)["pass"]
    bad_em = G.EMResult(200, 150, 140, 12, 2, G.mcnemar_one_sided(12, 2))       # 5-point drop, p ~ 0.006
    v = G.verdict(good, bad_em, noise)
    assert not v["pass"] and not v["checks"]["exact_match"]["ok"]
    noisy_em = G.EMResult(200, 150, 145, 6, 1, G.mcnemar_one_sided(6, 1))      # 2.5 points inside 3.0
    assert G.verdict(good, noisy_em, noise)["checks"]["exact_match"]["ok"]


def test_gate_end_to_end_tiny(capsys):
    G.main(["--model", "tiny_gqa", "--device", "cpu", "--test-kv", "fp8", "--ref-kv", "bf16", "--prompts", "6",
            "--len", "96", "--em-items", "6", "--em-answer", "4", "--calibrate"])
    import json
    rec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert rec["positions"] == 6 * 95 and rec["exact_match"]["items"] == 6
    assert rec["exact_match"]["control_correct"] == 6          # the control is the oracle: always right
    assert set(rec["verdict"]["checks"]) == {"kl_mean", "kl_p99", "top1", "dlogp_p99", "exact_match"}
    assert rec["noise"]["kl_mean"] >= 0.0
