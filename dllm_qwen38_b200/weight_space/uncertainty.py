"""Conservative paired-delta interval for a collected comparison bundle (supplementary to the
frozen bootstrap / McNemar numbers; the reference's `tools/weight-space/uncertainty.py:12-99` role).

For n paired problems with `wins` (candidate right, baseline wrong) and `losses` (the reverse),
the win and loss rates each get an exact two-sided binomial (Clopper-Pearson) interval at
confidence 1 - alpha/2; by the union (Bonferroni) bound both hold together with probability at
least 1 - alpha, whatever the dependence between them, so
    delta = p_win - p_loss  in  [win_lo - loss_hi, win_hi - loss_lo].
The binomial tails are summed in log space (lgamma) and inverted by bisection.

    python -m dllm_qwen38_b200.weight_space.uncertainty BUNDLE.json --output OUT.json
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import pathlib

MAX_N = 10000


def _log_binom_pmf(n: int, k: int, p: float) -> float:
    return (math.lgamma(n + 1) - math.lgamma(k + 1) - math.lgamma(n - k + 1) + k * math.log(p)
            + (n - k) * math.log1p(-p))


def binom_cdf(k: int, n: int, p: float) -> float:
    """P[X <= k] for X ~ Binomial(n, p)."""
    if k >= n or p <= 0.0:
        return 1.0
    if p >= 1.0:
        return 0.0
    return min(1.0, math.fsum(math.exp(_log_binom_pmf(n, i, p)) for i in range(k + 1)))


def _upper(k: int, n: int, tail: float) -> float:
    """Largest p with P[X <= k] >= tail (the exact upper limit for k successes)."""
    if k >= n:
        return 1.0
    if k == 0:  # closed form: (1 - p)^n = tail
        return -math.expm1(math.log(tail) / n)
    lo, hi = 0.0, 1.0
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if binom_cdf(k, n, mid) > tail:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def _check_conf(confidence: float) -> None:
    if not (isinstance(confidence, float) and math.isfinite(confidence) and 0.0 < confidence < 1.0):
        raise ValueError("confidence must be a float strictly between 0 and 1")


def binomial_interval(k: int, n: int, confidence: float = 0.95) -> list:
    """Exact two-sided interval for a binomial proportion with k successes of n."""
    if type(k) is not int or type(n) is not int or not (1 <= n <= MAX_N) or not (0 <= k <= n):
        raise ValueError(f"need integers 0 <= k <= n, 1 <= n <= {MAX_N}")
    _check_conf(confidence)
    tail = 0.5 * (1.0 - confidence)
    return [1.0 - _upper(n - k, n, tail), _upper(k, n, tail)]


def paired_interval(n: int, wins: int, losses: int, confidence: float = 0.95) -> dict:
    if any(type(x) is not int for x in (n, wins, losses)) or wins < 0 or losses < 0 or wins + losses > n:
        raise ValueError("invalid paired counts")
    _check_conf(confidence)
    marginal = 1.0 - 0.5 * (1.0 - confidence)
    w = binomial_interval(wins, n, marginal)
    lo = binomial_interval(losses, n, marginal)
    return {"n": n, "wins": wins, "losses": losses, "observed_delta": (wins - losses) / n,
            "confidence": confidence, "marginal_confidence": marginal, "win_interval": w, "loss_interval": lo,
            "interval": [w[0] - lo[1], w[1] - lo[0]]}


def analyze(bundle_path, confidence: float = 0.95) -> dict:
    path = pathlib.Path(bundle_path)
    raw = path.read_bytes()
    bundle = json.loads(raw)
    if bundle.get("schema") != "bdllm.ws.bundle/v1":
        raise ValueError("not a completed-run bundle from collect.py")
    out = []
    for pair in bundle["paired"]:
        res = pair["result"]
        n = res["baseline"]["n"]
        if res["candidate"]["n"] != n:
            raise ValueError("paired sizes differ")
        for name in (pair["baseline"], pair["candidate"]):
            ids = bundle["runs"][name]["identity"]["case_ids"]
            if len(ids) != n or len(set(ids)) != n:
                raise ValueError("case counts differ from the comparison")
        row = paired_interval(n, res["wins"], res["losses"], confidence)
        row.update(baseline=pair["baseline"], candidate=pair["candidate"],
                   frozen_bootstrap_interval=res["bootstrap_95_interval"],
                   frozen_mcnemar_p=res["mcnemar_exact_two_sided_p"])
        out.append(row)
    return {"schema": "bdllm.ws.uncertainty/v1", "source_bundle_sha256": hashlib.sha256(raw).hexdigest(),
            "analysis_code_sha256": hashlib.sha256(pathlib.Path(__file__).read_bytes()).hexdigest(),
            "method": "exact binomial (Clopper-Pearson) win and loss intervals at 1-alpha/2 each; "
                      "Bonferroni joint coverage; endpoints subtracted",
            "comparisons": out,
            "qualifications": ["supplementary: the frozen bootstrap and McNemar results are kept, not replaced",
                               "coverage assumes independent, identically distributed problem pairs",
                               "conservative, not a tight paired risk-difference interval",
                               "per comparison; no adjustment across comparisons"]}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("bundle", type=pathlib.Path)
    p.add_argument("--output", required=True, type=pathlib.Path)
    p.add_argument("--confidence", type=float, default=0.95)
    a = p.parse_args(argv)
    res = analyze(a.bundle, a.confidence)
    with a.output.open("x") as f:
        json.dump(res, f, indent=2)
        f.write("\n")
    print(json.dumps(res["comparisons"], indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
