"""Planner studies: scale search, catalogue cover + audit, and native-vs-joint comparisons.

* ``scale_case`` solves a free pool of ``n_long`` long and ``n_short`` short
  samples and reports the chosen microbatch shapes (reference:
  experiments/sequence_dynamic_cp/joint_cp_scale_search.py:17-74).
* ``catalogue_template`` / ``count_cover`` / ``audit_catalogue`` turn solved
  single-microbatch plans into a template catalogue, find the minimum-cost
  cover of a (long, short) count pair by dynamic programming over counts, then
  rebuild, re-score and memory-tie-break the assembled plan (reference:
  experiments/sequence_dynamic_cp/joint_cp_scale_audit.py:53-217). The cover
  recursion is the usual unbounded-knapsack DP over the two counts.
* ``native_vs_joint`` scores the native fixed-N scheduler at every capacity of
  a grid against the joint plan for the same pool and applies the
  memory/throughput preference (reference:
  experiments/sequence_dynamic_cp/joint_advantage_search.py and
  native_n_generalization_theory.py).
"""

from __future__ import annotations

import math
import time
from collections import Counter

from .joint.analysis import describe
from .joint.cost import Evaluator
from .joint.ir import Group, Layout, Microbatch, Plan, validate_plan
from .joint.memory_selection import prefer_lower_memory
from .joint.response import response_coverage
from .joint.solver import SearchOptions, solve
from .mixed import to_joint
from .native import replay as native_replay
from .onedim import from_rank_ids
from .policy import select as policy_select


# ---------------------------------------------------------------- scale search
def scale_case(n_long: int, long_len: int, n_short: int, short_len: int, world: int, pattern: str, model,
               options: SearchOptions | None = None) -> dict:
    values = [long_len] * n_long + [short_len] * n_short
    lengths = dict(enumerate(values))
    options = options or SearchOptions(beam=32, layouts=12, max_states=4_000_000, node_affinity=True,
                                       homogeneous_packing=True, balanced_packing=True, heavy_tail_packing=True)
    t0 = time.monotonic()
    result = solve(lengths, world, pattern, model, options)
    row = {"world": world, "input_samples": len(values), "input_tokens": sum(values), "status": result["status"],
           "wall_seconds": time.monotonic() - t0,
           "necessary_microbatch_token_ceiling": model.token_capacity_upper_bound(pattern, world)}
    if result["plan"] is None:
        return {"result": result, "row": row}
    plan = Plan.from_dict(result["plan"])
    shapes = Counter((sum(lengths[s] == long_len for g in b.ingress.groups for s in g.samples),
                      sum(lengths[s] == short_len for g in b.ingress.groups for s in g.samples))
                     for b in plan.microbatches)
    summary = describe(result, lengths, model)
    row.update({k: v for k, v in summary.items() if k not in ("batches", "stage_costs")})
    row["selected_microbatch_shapes"] = [{"long_samples": a, "short_samples": b, "microbatches": n}
                                         for (a, b), n in sorted(shapes.items())]
    return {"result": result, "row": row}


# ---------------------------------------------------------------- catalogue
def _relabel(batch: Microbatch, mapping: dict) -> Microbatch:
    def lay(layout):
        return Layout(tuple(Group(g.ranks, tuple(mapping[s] for s in g.samples)) for g in layout.groups),
                      layout.mode)
    return Microbatch(lay(batch.ingress), tuple((lay(a), lay(m)) for a, m in batch.layers))


def catalogue_template(plan: Plan, lengths: dict, long_len: int, short_len: int) -> list[dict]:
    """One template per microbatch: samples relabelled long-first, 0..n-1."""
    out = []
    for batch in plan.microbatches:
        ids = sorted({s for g in batch.ingress.groups for s in g.samples}, key=lambda s: (-lengths[s], s))
        mapping = {s: i for i, s in enumerate(ids)}
        vals = [lengths[s] for s in ids]
        if set(vals) - {long_len, short_len}:
            raise ValueError("catalogue templates hold only the two declared lengths")
        out.append({"plan": Plan(plan.world, plan.pattern, (_relabel(batch, mapping),)).to_dict(),
                    "long_samples": vals.count(long_len), "short_samples": vals.count(short_len)})
    return out


def count_cover(templates, n_long: int, n_short: int):
    """Minimum total cost of templates (long, short, cost, id) covering exactly the counts."""
    INF = math.inf
    best = [[INF] * (n_short + 1) for _ in range(n_long + 1)]
    back = [[None] * (n_short + 1) for _ in range(n_long + 1)]
    best[0][0] = 0.0
    for a in range(n_long + 1):
        for b in range(n_short + 1):
            here = best[a][b]
            if here == INF:
                continue
            for h, s, cost, tid in templates:
                if h + s <= 0:
                    raise ValueError("empty template")
                x, y = a + h, b + s
                if x <= n_long and y <= n_short and here + cost < best[x][y]:
                    best[x][y] = here + cost
                    back[x][y] = (h, s, tid)
    if best[n_long][n_short] == INF:
        raise ValueError("catalogue cannot cover the requested counts")
    chosen, a, b = [], n_long, n_short
    while a or b:
        h, s, tid = back[a][b]
        chosen.append(tid)
        a, b = a - h, b - s
    return best[n_long][n_short], chosen[::-1]


def audit_catalogue(catalogue: list[dict], n_long: int, long_len: int, n_short: int, short_len: int, world: int,
                    pattern: str, model, max_attention_cp: int | None = None,
                    memory_time_tolerance: float = 0.001) -> dict:
    templates = {}
    for index, row in enumerate(catalogue):
        plan = Plan.from_dict(row["plan"])
        if plan.world != world:
            raise ValueError("catalogue world mismatch")
        batch = plan.microbatches[0]
        if max_attention_cp and any(len(g.ranks) > max_attention_cp for a, _ in batch.layers for g in a.groups):
            continue
        h, s = row["long_samples"], row["short_samples"]
        ev = Evaluator(model, dict(enumerate([long_len] * h + [short_len] * s)), world, pattern).evaluate(batch)
        if ev["fits"] and ((h, s) not in templates or ev["predicted_ms"] < templates[h, s][2]):
            templates[h, s] = (h, s, ev["predicted_ms"], index)
    score, chosen = count_cover(list(templates.values()), n_long, n_short)
    lengths = dict(enumerate([long_len] * n_long + [short_len] * n_short))
    batches, next_long, next_short = [], 0, n_long
    for index in chosen:
        row = catalogue[index]
        h, s = row["long_samples"], row["short_samples"]
        ids = list(range(next_long, next_long + h)) + list(range(next_short, next_short + s))
        batches.append(_relabel(Plan.from_dict(row["plan"]).microbatches[0], dict(enumerate(ids))))
        next_long, next_short = next_long + h, next_short + s
    plan = Plan(world, pattern, tuple(batches))
    validate_plan(plan, lengths)
    ev = Evaluator(model, lengths, world, pattern)
    checks = [ev.evaluate(b) for b in batches]
    if not all(c["fits"] for c in checks) or not math.isclose(sum(c["predicted_ms"] for c in checks), score,
                                                            rel_tol=1e-12):
        raise AssertionError("catalogue cover and re-scored plan disagree")
    plan, memory = prefer_lower_memory(plan, lengths, model, memory_time_tolerance)
    validate_plan(plan, lengths)
    checks = [ev.evaluate(b) for b in plan.microbatches]
    total = sum(c["predicted_ms"] for c in checks) + model.update_ms
    result = {"world": world, "input_tokens": sum(lengths.values()), "input_samples": len(lengths),
              "plan": plan.to_dict(), "predicted_update_ms": total, "microbatch_evidence": checks,
              "status": "catalogue_incumbent_with_bounded_memory_selection_no_global_certificate",
              "memory_selection": memory, "catalogue_templates": len(catalogue), "usable_templates": len(templates),
              "selected_templates": [{"template": i, "microbatches": n} for i, n in sorted(Counter(chosen).items())],
              "cp_response_evidence": response_coverage(plan, lengths, model), "gpu_admitted": False,
              "state_budget_exhausted": False, "states_examined": None}
    result["analysis"] = describe(result, lengths, model)
    return result


# ---------------------------------------------------------------- native vs joint
def native_joint_plan(lengths: dict, world: int, pattern: str, capacity: int, min_cp: int = 1,
                      coalesce: bool = True) -> Plan:
    """The native fixed-N scheduler at token capacity ``capacity`` as a joint plan."""
    samples = sorted(lengths.items())
    rank_ids = native_replay(samples, world, capacity, min_cp)
    onedim = from_rank_ids(rank_ids)
    return to_joint(onedim, lengths, world, pattern, token_cap=capacity if coalesce else None)


def plan_score(plan: Plan, lengths: dict, model) -> dict:
    ev = Evaluator(model, lengths, plan.world, plan.pattern)
    checks = [ev.evaluate(b) for b in plan.microbatches]
    return {"time": sum(c["predicted_ms"] for c in checks) + model.update_ms,
            "peak": max(max(c["peak_bytes"]) for c in checks), "fits": all(c["fits"] for c in checks),
            "microbatches": len(plan.microbatches)}


def native_vs_joint(lengths: dict, world: int, pattern: str, model, capacities, reference_capacity: int,
                    alpha: float = 2.0, options: SearchOptions | None = None) -> dict:
    """Score native N at every capacity and the joint plan; apply the alpha rule against native N at
    ``reference_capacity``."""
    candidates = []
    for cap in sorted(set(capacities) | {reference_capacity}):
        try:
            plan = native_joint_plan(lengths, world, pattern, cap)
        except ValueError as err:
            candidates.append({"id": f"native_K{cap}", "kind": "native", "capacity": cap, "fits": False,
                               "time": math.inf, "peak": math.inf, "error": str(err)})
            continue
        candidates.append(dict(plan_score(plan, lengths, model), id=f"native_K{cap}", kind="native", capacity=cap))
    joint = solve(lengths, world, pattern, model, options or SearchOptions())
    if joint["plan"] is not None:
        jp = Plan.from_dict(joint["plan"])
        candidates.append(dict(plan_score(jp, lengths, model), id="joint", kind="joint"))
    usable = [c for c in candidates if math.isfinite(c["time"])]
    decision = policy_select(usable, f"native_K{reference_capacity}", alpha)
    ref = next(c for c in usable if c["id"] == f"native_K{reference_capacity}")
    best_native = min((c for c in usable if c["kind"] == "native" and c["fits"]), key=lambda c: c["time"])
    report = {"world": world, "pattern": pattern, "samples": len(lengths), "tokens": sum(lengths.values()),
              "candidates": candidates, "decision": decision,
              "joint_speedup_vs_reference": (ref["time"] / next(c["time"] for c in usable if c["id"] == "joint")
                                             if any(c["id"] == "joint" for c in usable) else None),
              "best_native_capacity": best_native["capacity"],
              "joint_speedup_vs_best_native": (best_native["time"] / next(c["time"] for c in usable
                                                                          if c["id"] == "joint")
                                               if any(c["id"] == "joint" for c in usable) else None)}
    return report


def report_markdown(report: dict) -> str:
    lines = [f"# Native N vs joint plan ({report['samples']} samples, {report['tokens']} tokens, "
             f"world {report['world']})", "", "| candidate | fits | predicted ms | peak GiB | microbatches |",
             "|---|---|---|---|---|"]
    for c in report["candidates"]:
        peak = c["peak"] / 2 ** 30 if math.isfinite(c["peak"]) else float("nan")
        lines.append(f"| {c['id']} | {c['fits']} | {c['time']:.2f} | {peak:.2f} | {c.get('microbatches', '-')} |")
    d = report["decision"]
    lines += ["", f"Selected: **{d['selected']}** ({d['selected_time']:.2f} ms); best native: {d['best_native']}; "
              f"frontier: {', '.join(d['physical_time_memory_frontier'])}."]
    return "\n".join(lines) + "\n"
