"""Bounded memory tie-break for homogeneous, rank-resident CP1 microbatches.

After the bounded search, the CP1 microbatches whose samples all have one
length, never leave their rank and put the same number of samples on every
rank form a family per length. Each family is repacked with a different number
of samples per rank (1 and ceil(i * widest / 16) for i = 1..16, so at most 17
candidates); a candidate replaces the family if the complete plan then has a
lower (peak, time) and its update time stays within ``1 + tolerance`` of the
original plan's (the tolerance is never compounded across families).
Distributed microbatches are never touched. Same rule and outputs as the
reference's joint_cp/memory_selection.py:14-96.
"""

from __future__ import annotations

import math

from .cost import Evaluator
from .ir import Group, Layout, Microbatch, Plan, validate_plan


class _Scorer:
    """(peak bytes, update ms, fits) of whole plans, memoised per microbatch."""

    def __init__(self, model, lengths: dict, world: int, pattern: str):
        self.ev = Evaluator(model, lengths, world, pattern)
        self.update_ms = model.update_ms
        self.rows: dict = {}

    def __call__(self, plan: Plan):
        rows = []
        for mb in plan.microbatches:
            row = self.rows.get(mb)
            if row is None:
                row = self.rows[mb] = self.ev.evaluate(mb)
            rows.append(row)
        peak = max(max(r["peak_bytes"]) for r in rows)
        ms = sum(r["predicted_ms"] for r in rows) + self.update_ms
        return peak, ms, all(r["fits"] for r in rows)


def _resident_length(mb: Microbatch, lengths: dict, world: int):
    """The common sample length if ``mb`` is CP1 everywhere, keeps every sample on its ingress
    rank in every layer and holds equally many samples per rank, else None."""
    owners = mb.ingress.rank_ids(world)
    layouts = [mb.ingress] + [x for pair in mb.layers for x in pair]
    if any(len(g.ranks) != 1 for x in layouts for g in x.groups):
        return None
    if any(x.rank_ids(world) != owners for x in layouts[1:]) or len({len(ids) for ids in owners}) != 1:
        return None
    sizes = {lengths[s] for ids in owners for s in ids}
    return sizes.pop() if len(sizes) == 1 else None


def _families(plan: Plan, lengths: dict) -> dict[int, list[int]]:
    out: dict[int, list[int]] = {}
    for i, mb in enumerate(plan.microbatches):
        length = _resident_length(mb, lengths, plan.world)
        if length is not None:
            out.setdefault(length, []).append(i)
    return out


def _repacked(queues: list[list[int]], count: int, pattern: str) -> list[Microbatch]:
    """The family's per-rank sample queues cut into microbatches of ``count`` samples per rank."""
    out = []
    for start in range(0, len(queues[0]), count):
        ingress = Layout(tuple(Group((r,), tuple(q[start:start + count])) for r, q in enumerate(queues)), "zigzag")
        flat = ingress.with_mode("contiguous")
        out.append(Microbatch(ingress, tuple((flat if c == "G" else ingress, flat) for c in pattern)))
    return out


def _spliced(plan: Plan, family: set, replacement: list[Microbatch]) -> Plan:
    """``plan`` with the family's microbatches replaced, in place of its first member."""
    batches, pending = [], True
    for mb in plan.microbatches:
        if mb not in family:
            batches.append(mb)
        elif pending:
            batches.extend(replacement)
            pending = False
    return Plan(plan.world, plan.pattern, tuple(batches))


def capacities_for(widest: int) -> list[int]:
    return sorted({1} | {-(-widest * i // 16) for i in range(1, 17)})


def prefer_lower_memory(plan: Plan, lengths: dict, model, relative_time_tolerance: float = 0.001):
    if not (math.isfinite(relative_time_tolerance) and relative_time_tolerance >= 0):
        raise ValueError("Memory selection requires a finite nonnegative time tolerance")
    validate_plan(plan, lengths)
    score = _Scorer(model, lengths, plan.world, plan.pattern)
    start_peak, start_ms, _ = score(plan)
    deadline = start_ms * (1 + relative_time_tolerance)
    selected, best = plan, (start_peak, start_ms)
    examined, changes = 0, []
    for length, members in sorted(_families(plan, lengths).items()):
        # members are named by the original microbatches, so earlier swaps cannot shift them
        family = {plan.microbatches[i] for i in members}
        queues = [[] for _ in range(plan.world)]
        for i in members:
            for r, ids in enumerate(plan.microbatches[i].ingress.rank_ids(plan.world)):
                queues[r] += ids
        widest = max(len(g.samples) for mb in family for g in mb.ingress.groups)
        winner, chosen = selected, None
        for count in capacities_for(widest):
            candidate = _spliced(selected, family, _repacked(queues, count, plan.pattern))
            peak, ms, fits = score(candidate)
            examined += 1
            if fits and ms <= deadline and (peak, ms) < best:
                winner, chosen, best = candidate, count, (peak, ms)
        selected = winner
        if chosen is not None:
            changes.append({"sample_length": length, "samples_per_rank": chosen, "tokens_per_rank": length * chosen})
    validate_plan(selected, lengths)
    return selected, {
        "policy": "min_peak_then_time_within_relative_update_tolerance",
        "relative_time_tolerance": relative_time_tolerance,
        "original_predicted_update_ms": start_ms, "selected_predicted_update_ms": best[1],
        "original_peak_bytes": start_peak, "selected_peak_bytes": best[0],
        "original_microbatches": len(plan.microbatches), "selected_microbatches": len(selected.microbatches),
        "candidates_examined": examined, "changed": selected != plan, "repacked_families": changes,
        "scope": "bounded homogeneous rank-resident CP1 repacking; distributed batches unchanged",
        "global_optimality_certificate": False}
