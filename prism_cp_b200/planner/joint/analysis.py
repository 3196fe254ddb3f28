"""Stage accounting of a solved plan, and re-scoring of arbitrary plans.

``describe`` walks a solved plan once with the evaluator and books every priced
piece into one of six stages (GDN, GQA, MLP, routes, head plus per-microbatch
overhead, update); the stages must add up to the plan's score, which guards
against the solver and the evaluator drifting apart. It also summarises each
microbatch: samples, input tokens, and per layer the CP degree of every sample
length and the largest per-rank token counts. ``measure`` re-scores any plan.
Same outputs as the reference's joint_cp/analysis.py:10-54.
"""

from __future__ import annotations

import math
from collections import Counter

from .cost import Evaluator, resource_metrics
from .ir import Plan, validate_plan

STAGES = ("gdn_ms", "gqa_ms", "mlp_ms", "routes_ms", "head_and_mb_ms", "update_ms")


class _Ledger:
    def __init__(self, update_ms: float):
        self.ms = dict.fromkeys(STAGES, 0.0)
        self.ms["update_ms"] = update_ms

    def book(self, stage: str, ms: float) -> None:
        self.ms[stage] += ms

    def total(self) -> float:
        return sum(self.ms.values())


def _layer_summary(symbol, attention, mlp, lengths, world) -> dict:
    per_shape = Counter((lengths[s], cp) for s, cp in attention.sample_cp())
    return {"operator": "GDN" if symbol == "G" else "GQA",
            "cp_by_length": [{"length": n, "cp": cp, "samples": k} for (n, cp), k in sorted(per_shape.items())],
            "max_attention_tokens": max(attention.tokens(lengths, world)),
            "max_mlp_tokens": max(mlp.tokens(lengths, world))}


def _book_microbatch(ev: Evaluator, ledger: _Ledger, mb, pattern: str) -> None:
    current = mb.ingress
    for symbol, (attention, mlp) in zip(pattern, mb.layers):
        ledger.book("gdn_ms" if symbol == "G" else "gqa_ms", ev.operator(symbol, attention)[0])
        ledger.book("mlp_ms", ev.operator("M", mlp)[0])
        ledger.book("routes_ms", ev.transfer(current, attention)[0] + 2 * ev.transfer(attention, mlp)[0])
        current = attention
    finish_ms, _ = ev.finish(ev.initial(mb.ingress), current, mb.ingress)
    home = ev.transfer(current, mb.ingress)[0]
    ledger.book("routes_ms", home)
    ledger.book("head_and_mb_ms", finish_ms - home)


def describe(result: dict, lengths: dict, model) -> dict:
    if result["plan"] is None:
        return {"status": result["status"]}
    plan = Plan.from_dict(result["plan"])
    ev = Evaluator(model, lengths, plan.world, plan.pattern)
    ledger = _Ledger(model.update_ms)
    batches = []
    for mb in plan.microbatches:
        _book_microbatch(ev, ledger, mb, plan.pattern)
        samples = [s for g in mb.ingress.groups for s in g.samples]
        batches.append({"samples": len(samples), "input_tokens": sum(lengths[s] for s in samples),
                        "layers": [_layer_summary(sym, a, m, lengths, plan.world)
                                   for sym, (a, m) in zip(plan.pattern, mb.layers)],
                        "changes_cp": len({a.sample_cp() for a, _ in mb.layers}) > 1})
    predicted = result["predicted_update_ms"]
    if not math.isclose(ledger.total(), predicted, rel_tol=1e-10, abs_tol=1e-8):
        raise AssertionError("Stage breakdown does not match the complete plan score")
    peak = max(max(e["peak_bytes"]) for e in result["microbatch_evidence"])
    return {"status": result["status"], "predicted_update_ms": predicted,
            "resource_metrics": resource_metrics(lengths, plan.world, plan.pattern, model, predicted),
            "microbatches": len(batches), "changed_cp_microbatches": sum(b["changes_cp"] for b in batches),
            "peak_gib": peak / 1024 ** 3, "stage_costs": ledger.ms, "batches": batches,
            "state_budget_exhausted": result["state_budget_exhausted"], "states_examined": result["states_examined"]}


def measure(plan: Plan, lengths: dict, model):
    """(predicted update ms, per-microbatch evidence) of any valid plan."""
    validate_plan(plan, lengths)
    ev = Evaluator(model, lengths, plan.world, plan.pattern)
    evidence = [ev.evaluate(b) for b in plan.microbatches]
    return model.update_ms + sum(e["predicted_ms"] for e in evidence), evidence
