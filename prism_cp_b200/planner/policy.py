"""Memory/throughput preference and the variable-capacity (per-batch K) rule.

The rules (same inputs give the same decisions as the reference's
memory_performance_policy.py:11-54 and random_batch_capacity_analysis.py:25-100):

* A candidate that grows the memory peak by a fraction ``m`` over a common
  reference is worth it only if its throughput gain ``g`` is at least
  ``alpha * m`` (alpha = 2 by default); a candidate that does not grow memory
  needs no gain; a physically infeasible candidate is never accepted.
* Among accepted candidates the winner minimises (time, peak, not-the-reference,
  id); the Pareto frontier of the feasible (peak, time) points is reported.
* Per-batch capacity K: a fixed reference K plus every length's CP threshold
  ceil32(L / p) over dyadic p, kept inside a declared window.
* Over a finite batch distribution the expected update time of the fixed-K,
  per-batch-K, finite-oracle and selected policies is a ratio of expectations.

Structure: a decision is a small value object; a candidate table is ranked by
one key function; the frontier is a single sweep over points sorted by peak.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

ALIGNMENT, FIXED_REFERENCE = 32, 16 * 1024
TIME, PEAK = "predicted_update_ms", "peak_gib"


@dataclass(frozen=True)
class Decision:
    """Outcome of comparing one candidate against the reference."""

    fits: bool
    growth: float       # fractional memory growth over the reference
    gain: float         # fractional throughput gain over the reference
    required: float     # gain the growth demands

    @property
    def worth_growth(self) -> bool:
        return (self.growth <= 0 or self.gain >= self.required
                or math.isclose(self.gain, self.required, abs_tol=1e-12))

    @property
    def reason(self) -> str:
        if not self.fits:
            return "physical_memory_rejected"
        if not self.worth_growth:
            return "insufficient_throughput_gain"
        return "no_memory_increase" if self.growth <= 0 else "gain_covers_memory_growth"

    def as_dict(self) -> dict:
        return {"accepted": bool(self.fits and self.worth_growth), "reason": self.reason,
                "memory_growth_pct": 100 * self.growth, "throughput_gain_pct": 100 * self.gain,
                "required_throughput_gain_pct": 100 * self.required}


def _check_positive(*values) -> None:
    for v in values:
        if not (math.isfinite(v) and v > 0):
            raise ValueError("Times and memory peaks must be finite and positive")


def tradeoff(reference_time, reference_peak, candidate_time, candidate_peak, *, min_gain_per_memory_growth=2.0,
             fits=True) -> dict:
    _check_positive(reference_time, reference_peak, candidate_time, candidate_peak)
    alpha = min_gain_per_memory_growth
    if not (math.isfinite(alpha) and alpha >= 0):
        raise ValueError("The gain multiplier must be finite and nonnegative")
    growth = candidate_peak / reference_peak - 1
    d = Decision(bool(fits), growth, reference_time / candidate_time - 1, alpha * max(0.0, growth))
    return d.as_dict()


def pareto_frontier(points: list[dict]) -> list[str]:
    """Ids of the (peak, time) points no other point dominates, in (peak, time) order.
    Identical points do not dominate each other, so duplicates of a frontier point stay."""
    out, best_time, last = [], math.inf, None
    for c in sorted(points, key=lambda c: (c["peak"], c["time"])):
        here = (c["peak"], c["time"])
        if c["time"] < best_time or here == last:
            out.append(c["id"])
            best_time, last = min(best_time, c["time"]), here
    return out


def select(candidates: list[dict], reference_id: str, multiplier: float = 2.0) -> dict:
    by_id = {c["id"]: c for c in reversed(candidates)}
    ref = by_id[reference_id]
    if not ref["fits"]:
        raise ValueError("The common reference must be physically feasible")
    table = []
    for c in candidates:
        decision = tradeoff(ref["time"], ref["peak"], c["time"], c["peak"], min_gain_per_memory_growth=multiplier,
                            fits=c["fits"])
        table.append({**c, "decision": decision})

    def rank(c):
        return c["time"], c["peak"], c["id"] != reference_id, c["id"]

    accepted = sorted((c for c in table if c["decision"]["accepted"]), key=rank)
    native = next((c for c in accepted if c["kind"] == "native"), None)
    if native is None:
        raise ValueError("no native candidate is accepted")
    return {"reference": reference_id, "candidates": table, "best_native": native["id"],
            "best_native_time": native["time"], "selected": accepted[0]["id"], "selected_time": accepted[0]["time"],
            "physical_time_memory_frontier": pareto_frontier([c for c in table if c["fits"]])}


def capacity_shortlist(lengths, reference: int = FIXED_REFERENCE, world: int = 16,
                       lo: int = 8 * 1024, hi: int = 40 * 1024) -> list[int]:
    """Per-rank capacities K (multiples of 32 tokens, not powers of two) inside [lo, hi]:
    the reference K and, for every distinct length, the smallest K that fits it at each
    dyadic CP degree up to ``world``."""
    degrees = [1 << e for e in range(world.bit_length()) if (1 << e) <= world]
    floor = max(lo, -(-max(lengths) // world))
    thresholds = {ALIGNMENT * -(-n // (p * ALIGNMENT)) for n in set(lengths) for p in degrees}
    return sorted(k for k in thresholds | {reference} if floor <= k <= hi)


# ------------------------------------------------------------------ per-batch K over a batch law
def is_eligible(score, reference, preference) -> bool:
    if not score["model_fits"]:
        return False
    if preference == "physical":
        return True
    return tradeoff(reference[TIME], reference[PEAK], score[TIME], score[PEAK],
                    min_gain_per_memory_growth=2.0)["accepted"]


class _Case:
    """One cached batch shape scored under one CP-response policy."""

    def __init__(self, case: dict, policy: str, preference: str):
        self.case, self.policy = case, policy
        self.ref = next(n["scores"][policy] for n in case["native"] if n["capacity_tokens"] == FIXED_REFERENCE)
        ok = lambda row: is_eligible(row["scores"][policy], self.ref, preference)  # noqa: E731
        self.native = [n for n in case["native"] if ok(n)]
        self.joint = [j for j in case["joint"] if ok(j)]

    def key(self, row):
        s = row["scores"][self.policy]
        return s[TIME], s[PEAK], row["id"]

    def best(self, rows):
        rows = list(rows)
        return min(rows, key=self.key) if rows else None

    def compact(self, row):
        if row is None:
            return None
        s = row["scores"][self.policy]
        return {"id": row["id"], "capacity_tokens": row.get("capacity_tokens"), "time_ms": s[TIME],
                "peak_gib": s[PEAK]}


def choose(case, policy, preference) -> dict:
    c = _Case(case, policy, preference)
    simple = c.best(n for n in c.native if n["capacity_tokens"] in case["simple_capacity_tokens"])
    oracle = c.best(c.native)
    best_joint = c.best(c.joint)
    chosen = c.best([simple, *c.joint])
    t = lambda row: row["scores"][policy][TIME]  # noqa: E731
    return {"simple": c.compact(simple), "finite_oracle": c.compact(oracle), "best_joint": c.compact(best_joint),
            "selected": c.compact(chosen), "feasible_native": {n["capacity_tokens"]: c.compact(n) for n in c.native},
            "simple_matches_finite_oracle": math.isclose(t(simple), t(oracle), rel_tol=1e-12)}


def _expectation(weighted: list[tuple[float, dict]], tokens: float) -> dict:
    mean = sum(w * e["time_ms"] for w, e in weighted)
    return {"expected_update_ms": mean, "effective_tokens_per_second": 1000 * tokens / mean,
            "worst_case_model_peak_gib": max(e["peak_gib"] for _, e in weighted)}


def integrate(cases, weights, policy, preference) -> dict:
    """Expected update time of each capacity policy over a finite batch law (ratio of expectations)."""
    law = [(c, weights[c["case"]]) for c in cases if weights.get(c["case"], 0.0) > 0]
    if not math.isclose(sum(w for _, w in law), 1.0):
        raise ValueError("case weights must sum to one")
    picks = [(w, choose(c, policy, preference)) for c, w in law]
    shared = set.intersection(*(set(d["feasible_native"]) for _, d in picks))
    expected_fixed = {k: sum(w * d["feasible_native"][k]["time_ms"] for w, d in picks) for k in shared}
    fixed_k = min(shared, key=lambda k: (expected_fixed[k], k))
    tokens = sum(w * c["input_tokens"] for c, w in law)
    out = {"fixed_capacity_tokens": fixed_k, "weights": weights, "expected_tokens": tokens}
    out["fixed"] = _expectation([(w, d["feasible_native"][fixed_k]) for w, d in picks], tokens)
    for method in ("simple", "finite_oracle", "selected"):
        out[method] = _expectation([(w, d[method]) for w, d in picks], tokens)
    fixed, adapt, joint = expected_fixed[fixed_k], out["simple"]["expected_update_ms"], \
        out["selected"]["expected_update_ms"]
    out.update(simple_gain_vs_fixed_pct=100 * (fixed / adapt - 1),
               selection_gain_vs_simple_pct=100 * (adapt / joint - 1),
               selection_gain_vs_fixed_pct=100 * (fixed / joint - 1),
               capacity_saving_ms=fixed - adapt, additional_joint_saving_ms=adapt - joint,
               joint_selected_probability=sum(w for w, d in picks if d["selected"]["id"].startswith("J_")),
               simple_matches_finite_oracle=all(d["simple_matches_finite_oracle"] for _, d in picks))
    return out
