"""Memory/throughput preference and the variable-capacity (per-batch K) rule.

* ``tradeoff`` / ``select``: accept a memory growth ``m`` only when the
  throughput gain ``g >= alpha * m`` (alpha = 2 by default); symmetric for native
  and joint candidates; physical feasibility always wins; the raw
  time/memory Pareto frontier is reported (reference:
  memory_performance_policy.py:11-54).
* ``capacity_shortlist``: candidate per-rank capacities K for a global batch -
  a fixed reference K plus each length's CP threshold ceil32(L / p) for
  p in 1..16, kept within 8..40Ki (reference: random_batch_capacity_analysis.py:25-35).
* ``integrate``: expected update time of fixed-K / per-batch-K / oracle /
  selected policies over a finite batch distribution as a ratio of
  expectations, never a mean of per-batch ratios (reference: :50-100).
"""

from __future__ import annotations

import math

ALIGNMENT, FIXED_REFERENCE = 32, 16 * 1024


def tradeoff(reference_time, reference_peak, candidate_time, candidate_peak, *, min_gain_per_memory_growth=2.0,
             fits=True) -> dict:
    vals = (reference_time, reference_peak, candidate_time, candidate_peak)
    if any(not math.isfinite(v) or v <= 0 for v in vals):
        raise ValueError("Times and memory peaks must be finite and positive")
    if not math.isfinite(min_gain_per_memory_growth) or min_gain_per_memory_growth < 0:
        raise ValueError("The gain multiplier must be finite and nonnegative")
    growth = candidate_peak / reference_peak - 1
    gain = reference_time / candidate_time - 1
    required = min_gain_per_memory_growth * max(0.0, growth)
    worth = growth <= 0 or gain >= required or math.isclose(gain, required, abs_tol=1e-12)
    reason = ("physical_memory_rejected" if not fits else "insufficient_throughput_gain" if not worth
              else "no_memory_increase" if growth <= 0 else "gain_covers_memory_growth")
    return {"accepted": bool(fits and worth), "reason": reason, "memory_growth_pct": 100 * growth,
            "throughput_gain_pct": 100 * gain, "required_throughput_gain_pct": 100 * required}


def select(candidates: list[dict], reference_id: str, multiplier: float = 2.0) -> dict:
    ref = next(c for c in candidates if c["id"] == reference_id)
    if not ref["fits"]:
        raise ValueError("The common reference must be physically feasible")
    rows = [dict(c, decision=tradeoff(ref["time"], ref["peak"], c["time"], c["peak"],
                                      min_gain_per_memory_growth=multiplier, fits=c["fits"])) for c in candidates]
    ok = [c for c in rows if c["decision"]["accepted"]]
    key = lambda c: (c["time"], c["peak"], c["id"] != reference_id, c["id"])
    best_native = min((c for c in ok if c["kind"] == "native"), key=key)
    chosen = min(ok, key=key)
    feasible = [c for c in rows if c["fits"]]
    frontier = [c["id"] for c in sorted(feasible, key=lambda c: (c["peak"], c["time"]))
                if not any(d["peak"] <= c["peak"] and d["time"] <= c["time"]
                           and (d["peak"] < c["peak"] or d["time"] < c["time"]) for d in feasible)]
    return {"reference": reference_id, "candidates": rows, "best_native": best_native["id"],
            "best_native_time": best_native["time"], "selected": chosen["id"], "selected_time": chosen["time"],
            "physical_time_memory_frontier": frontier}


def capacity_shortlist(lengths, reference: int = FIXED_REFERENCE, world: int = 16,
                       lo: int = 8 * 1024, hi: int = 40 * 1024) -> list[int]:
    """K values aligned to 32 tokens (not powers of two), within [lo, hi]."""
    minimum = math.ceil(max(lengths) / world)
    values = {reference}
    cps = []
    p = 1
    while p <= world:
        cps.append(p)
        p *= 2
    values.update(math.ceil(n / (cp * ALIGNMENT)) * ALIGNMENT for n in set(lengths) for cp in cps)
    return sorted(k for k in values if max(lo, minimum) <= k <= hi)


def is_eligible(score, reference, preference):
    return score["model_fits"] and (preference == "physical" or tradeoff(
        reference["predicted_update_ms"], reference["peak_gib"], score["predicted_update_ms"], score["peak_gib"],
        min_gain_per_memory_growth=2.0)["accepted"])


def choose(case, policy, preference):
    ref = next(n["scores"][policy] for n in case["native"] if n["capacity_tokens"] == FIXED_REFERENCE)
    native = [n for n in case["native"] if is_eligible(n["scores"][policy], ref, preference)]
    key = lambda r: (r["scores"][policy]["predicted_update_ms"], r["scores"][policy]["peak_gib"], r["id"])
    simple = min((n for n in native if n["capacity_tokens"] in case["simple_capacity_tokens"]), key=key)
    oracle = min(native, key=key)
    joint = [j for j in case["joint"] if is_eligible(j["scores"][policy], ref, preference)]
    best_joint = min(joint, key=key) if joint else None
    chosen = min([simple, *joint], key=key)

    def compact(row):
        if row is None:
            return None
        s = row["scores"][policy]
        return {"id": row["id"], "capacity_tokens": row.get("capacity_tokens"), "time_ms": s["predicted_update_ms"],
                "peak_gib": s["peak_gib"]}

    return {"simple": compact(simple), "finite_oracle": compact(oracle), "best_joint": compact(best_joint),
            "selected": compact(chosen), "feasible_native": {n["capacity_tokens"]: compact(n) for n in native},
            "simple_matches_finite_oracle": math.isclose(simple["scores"][policy]["predicted_update_ms"],
                                                         oracle["scores"][policy]["predicted_update_ms"],
                                                         rel_tol=1e-12)}


def integrate(cases, weights, policy, preference) -> dict:
    active = [(c, weights.get(c["case"], 0.0)) for c in cases if weights.get(c["case"], 0.0) > 0]
    if not math.isclose(sum(w for _, w in active), 1.0):
        raise ValueError("case weights must sum to one")
    decisions = [(c, w, choose(c, policy, preference)) for c, w in active]
    common = set.intersection(*(set(d["feasible_native"]) for _, _, d in decisions))
    fixed_k = min(common, key=lambda k: (sum(w * d["feasible_native"][k]["time_ms"] for _, w, d in decisions), k))
    fixed_time = sum(w * d["feasible_native"][fixed_k]["time_ms"] for _, w, d in decisions)
    out = {"fixed_capacity_tokens": fixed_k, "weights": weights,
           "expected_tokens": sum(w * c["input_tokens"] for c, w in active)}
    for method in ("fixed", "simple", "finite_oracle", "selected"):
        entries = [(w, d["feasible_native"][fixed_k] if method == "fixed" else d[method]) for _, w, d in decisions]
        mean = sum(w * e["time_ms"] for w, e in entries)
        out[method] = {"expected_update_ms": mean,
                       "effective_tokens_per_second": 1000 * out["expected_tokens"] / mean,
                       "worst_case_model_peak_gib": max(e["peak_gib"] for _, e in entries)}
    adapt, joint = out["simple"]["expected_update_ms"], out["selected"]["expected_update_ms"]
    out.update(simple_gain_vs_fixed_pct=100 * (fixed_time / adapt - 1),
               selection_gain_vs_simple_pct=100 * (adapt / joint - 1),
               selection_gain_vs_fixed_pct=100 * (fixed_time / joint - 1),
               capacity_saving_ms=fixed_time - adapt, additional_joint_saving_ms=adapt - joint,
               joint_selected_probability=sum(w for _, w, d in decisions if d["selected"]["id"].startswith("J_")),
               simple_matches_finite_oracle=all(d["simple_matches_finite_oracle"] for _, _, d in decisions))
    return out
