"""Stage accounting of a solved plan and re-scoring of arbitrary plans.

``describe`` splits the predicted update into GDN, GQA, MLP, routes, head and
per-microbatch overhead, and update, and asserts the parts add up to the
plan's score (reference: joint_cp/analysis.py:10-47). ``measure`` re-scores a
plan under a model (reference: joint_cp/analysis.py:50-54).
"""

from __future__ import annotations

import math
from collections import Counter

from .cost import Evaluator, resource_metrics
from .ir import Plan, validate_plan


def describe(result: dict, lengths: dict, model) -> dict:
    if result["plan"] is None:
        return {"status": result["status"]}
    plan = Plan.from_dict(result["plan"])
    ev = Evaluator(model, lengths, plan.world, plan.pattern)
    costs = {"gdn_ms": 0.0, "gqa_ms": 0.0, "mlp_ms": 0.0, "routes_ms": 0.0, "head_and_mb_ms": 0.0,
             "update_ms": model.update_ms}
    batches = []
    for mb in plan.microbatches:
        prev = mb.ingress
        layers = []
        for symbol, (att, mlp) in zip(plan.pattern, mb.layers):
            costs["gdn_ms" if symbol == "G" else "gqa_ms"] += ev.operator(symbol, att)[0]
            costs["mlp_ms"] += ev.operator("M", mlp)[0]
            costs["routes_ms"] += ev.transfer(prev, att)[0] + 2 * ev.transfer(att, mlp)[0]
            counts = Counter((lengths[s], cp) for s, cp in att.sample_cp())
            layers.append({"operator": "GDN" if symbol == "G" else "GQA",
                           "cp_by_length": [{"length": n, "cp": cp, "samples": c}
                                            for (n, cp), c in sorted(counts.items())],
                           "max_attention_tokens": max(att.tokens(lengths, plan.world)),
                           "max_mlp_tokens": max(mlp.tokens(lengths, plan.world))})
            prev = att
        head, _ = ev.finish(ev.initial(mb.ingress), prev, mb.ingress)
        back = ev.transfer(prev, mb.ingress)[0]
        costs["routes_ms"] += back
        costs["head_and_mb_ms"] += head - back
        ids = [s for g in mb.ingress.groups for s in g.samples]
        batches.append({"samples": len(ids), "input_tokens": sum(lengths[s] for s in ids), "layers": layers,
                        "changes_cp": len({a.sample_cp() for a, _ in mb.layers}) > 1})
    predicted = result["predicted_update_ms"]
    if not math.isclose(sum(costs.values()), predicted, rel_tol=1e-10, abs_tol=1e-8):
        raise AssertionError("Stage breakdown does not match the complete plan score")
    return {"status": result["status"], "predicted_update_ms": predicted,
            "resource_metrics": resource_metrics(lengths, plan.world, plan.pattern, model, predicted),
            "microbatches": len(batches), "changed_cp_microbatches": sum(b["changes_cp"] for b in batches),
            "peak_gib": max(max(e["peak_bytes"]) for e in result["microbatch_evidence"]) / 1024 ** 3,
            "stage_costs": costs, "batches": batches,
            "state_budget_exhausted": result["state_budget_exhausted"], "states_examined": result["states_examined"]}


def measure(plan: Plan, lengths: dict, model):
    validate_plan(plan, lengths)
    ev = Evaluator(model, lengths, plan.world, plan.pattern)
    evidence = [ev.evaluate(b) for b in plan.microbatches]
    return sum(e["predicted_ms"] for e in evidence) + model.update_ms, evidence
