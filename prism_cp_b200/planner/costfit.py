"""CP1 module cost fit and domain-checked query.

Fits measured single-GPU (CP = 1) forward+backward times of one module against
``(S^2, S, 1)`` (attention-like) or ``(S, 1)`` (linear) features with
non-negative coefficients, and reports held-out errors. The non-negative least
squares problem is solved exactly by enumerating active sets: for the two or
three features used here every subset is solved by ordinary least squares and
the best feasible (all coefficients >= 0) subset wins, which is the global
NNLS optimum. Behaviour follows the reference fit
(experiments/performance_model/fit_costs.py:12-119) and its query, which
refuses any CP other than 1 (experiments/performance_model/cost_model.py:6-35).
"""

from __future__ import annotations

import argparse
import itertools
import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path

import numpy as np

FEATURES = {"quadratic": ("S2", "S", "1"), "linear": ("S", "1")}


def _design(lengths, kind: str) -> np.ndarray:
    s = np.asarray(lengths, dtype=np.float64)
    cols = {"S2": s * s, "S": s, "1": np.ones_like(s)}
    return np.stack([cols[f] for f in FEATURES[kind]], axis=1)


def nnls_exact(A: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Global non-negative least squares by active-set enumeration (few columns)."""
    n = A.shape[1]
    if n > 8:
        raise ValueError("exact enumeration is meant for a handful of features")
    best, best_res = np.zeros(n), float(np.sum(b * b))
    for r in range(1, n + 1):
        for cols in itertools.combinations(range(n), r):
            sub = A[:, cols]
            coef, *_ = np.linalg.lstsq(sub, b, rcond=None)
            if np.any(coef < 0):
                continue
            res = float(np.sum((sub @ coef - b) ** 2))
            if res < best_res - 1e-15 * max(1.0, best_res):
                best = np.zeros(n)
                best[list(cols)] = coef
                best_res = res
    return best


@dataclass(frozen=True)
class CostFit:
    module: str
    kind: str
    coefficients: dict
    domain_tokens: tuple
    train_points: int
    holdout_points: int
    holdout_max_relative_error: float | None
    holdout_mean_relative_error: float | None

    def query(self, tokens: int, cp: int = 1) -> float:
        """Predicted F+B milliseconds at ``tokens`` on one GPU; refuses CP != 1 and out-of-domain lengths."""
        if cp != 1:
            raise ValueError("the CP1 cost fit cannot price CP > 1; use a measured CP response profile")
        lo, hi = self.domain_tokens
        if not lo <= tokens <= hi:
            raise ValueError(f"{tokens} tokens is outside the fitted domain [{lo}, {hi}]")
        x = _design([tokens], self.kind)[0]
        return float(sum(self.coefficients[f] * v for f, v in zip(FEATURES[self.kind], x)))


def fit(module: str, lengths, milliseconds, kind: str = "quadratic", holdout_every: int = 0) -> CostFit:
    """Fit one module's CP1 times; every ``holdout_every``-th point (if > 0) is held out."""
    lengths = [int(x) for x in lengths]
    ms = [float(x) for x in milliseconds]
    if len(lengths) != len(ms) or not lengths:
        raise ValueError("need matching, non-empty length/time lists")
    if any(not math.isfinite(t) or t <= 0 for t in ms):
        raise ValueError("times must be finite and positive")
    idx = list(range(len(lengths)))
    hold = [i for i in idx if holdout_every > 0 and i % holdout_every == holdout_every - 1]
    train = [i for i in idx if i not in hold]
    A = _design([lengths[i] for i in train], kind)
    b = np.asarray([ms[i] for i in train])
    coef = nnls_exact(A, b)
    coefficients = dict(zip(FEATURES[kind], (float(c) for c in coef)))
    errs = []
    for i in hold:
        pred = float(_design([lengths[i]], kind)[0] @ coef)
        errs.append(abs(pred - ms[i]) / ms[i])
    return CostFit(module, kind, coefficients, (min(lengths), max(lengths)), len(train), len(hold),
                   max(errs) if errs else None, float(np.mean(errs)) if errs else None)


def fit_records(records: list[dict], holdout_every: int = 4) -> dict[str, CostFit]:
    """Fit every module of module-bench records (``cp == 1`` rows only)."""
    by_module: dict[str, list] = {}
    for r in records:
        if int(r.get("cp", 1)) == 1:
            by_module.setdefault(r["module"], []).append((int(r["tokens"]), float(r["fb_ms"])))
    out = {}
    for module, pts in sorted(by_module.items()):
        pts.sort()
        kind = "quadratic" if module in ("GQA", "GDN") else "linear"
        out[module] = fit(module, [p[0] for p in pts], [p[1] for p in pts], kind, holdout_every)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description="Fit CP1 module costs from module-bench records")
    ap.add_argument("--records", type=Path, required=True, help="module bench JSON (list of records)")
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--holdout-every", type=int, default=4)
    args = ap.parse_args(argv)
    data = json.loads(args.records.read_text())
    records = data["records"] if isinstance(data, dict) else data
    fits = fit_records(records, args.holdout_every)
    args.output.write_text(json.dumps({m: asdict(f) for m, f in fits.items()}, indent=2) + "\n")
    print(json.dumps({m: f.coefficients for m, f in fits.items()}))


if __name__ == "__main__":
    main()
