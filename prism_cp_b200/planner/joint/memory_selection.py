"""Bounded memory tie-break for homogeneous, rank-resident CP1 microbatches.

After the bounded search, families of CP1 microbatches whose samples all have
one length and never leave their rank are repacked with fewer or more samples
per rank (at most 17 candidate capacities per family: 1 and ceil(i*max/16)),
keeping the candidate with the lowest peak memory whose complete update time
stays within ``(1 + tolerance)`` of the original. Distributed microbatches are
never touched. Same rule as the reference
(experiments/sequence_dynamic_cp/joint_cp/memory_selection.py:14-96).
"""

from __future__ import annotations

import math

from .cost import Evaluator
from .ir import Group, Layout, Microbatch, Plan, validate_plan


def prefer_lower_memory(plan: Plan, lengths: dict, model, relative_time_tolerance: float = 0.001):
    if not math.isfinite(relative_time_tolerance) or relative_time_tolerance < 0:
        raise ValueError("Memory selection requires a finite nonnegative time tolerance")
    validate_plan(plan, lengths)
    ev = Evaluator(model, lengths, plan.world, plan.pattern)
    memo: dict = {}

    def score(candidate: Plan):
        rows = []
        for mb in candidate.microbatches:
            if mb not in memo:
                memo[mb] = ev.evaluate(mb)
            rows.append(memo[mb])
        return (max(max(r["peak_bytes"]) for r in rows), sum(r["predicted_ms"] for r in rows) + model.update_ms,
                all(r["fits"] for r in rows))

    peak0, ms0, _ = score(plan)
    deadline = ms0 * (1 + relative_time_tolerance)
    selected, best = plan, score(plan)
    families: dict[int, list[int]] = {}
    for i, mb in enumerate(plan.microbatches):
        owners = mb.ingress.rank_ids(plan.world)
        layouts = [mb.ingress, *(x for pair in mb.layers for x in pair)]
        if (any(len(g.ranks) != 1 for x in layouts for g in x.groups)
                or any(x.rank_ids(plan.world) != owners for x in layouts)
                or len({len(r) for r in owners}) != 1):
            continue
        sizes = {lengths[s] for r in owners for s in r}
        if len(sizes) == 1:
            families.setdefault(next(iter(sizes)), []).append(i)
    examined, changes = 0, []
    for length, indices in sorted(families.items()):
        old = {plan.microbatches[i] for i in indices}
        queues: list[list[int]] = [[] for _ in range(plan.world)]
        for i in indices:
            for r, ids in enumerate(plan.microbatches[i].ingress.rank_ids(plan.world)):
                queues[r].extend(ids)
        widest = max(len(g.samples) for b in old for g in b.ingress.groups)
        capacities = sorted({1, *((widest * i + 15) // 16 for i in range(1, 17))})
        family_best, chosen = selected, None
        for count in capacities:
            replacement = []
            for start in range(0, len(queues[0]), count):
                groups = tuple(Group((r,), tuple(ids[start:start + count])) for r, ids in enumerate(queues))
                ingress = Layout(groups, "zigzag")
                contiguous = ingress.with_mode("contiguous")
                replacement.append(Microbatch(ingress, tuple((contiguous if c == "G" else ingress, contiguous)
                                                             for c in plan.pattern)))
            batches, placed = [], False
            for mb in selected.microbatches:
                if mb in old:
                    if not placed:
                        batches.extend(replacement)
                        placed = True
                else:
                    batches.append(mb)
            candidate = Plan(plan.world, plan.pattern, tuple(batches))
            peak, ms, fits = score(candidate)
            examined += 1
            if fits and ms <= deadline and (peak, ms) < best[:2]:
                family_best, chosen = candidate, count
                best = (peak, ms, fits)
        selected = family_best
        if chosen is not None:
            changes.append({"sample_length": length, "samples_per_rank": chosen, "tokens_per_rank": length * chosen})
    validate_plan(selected, lengths)
    return selected, {
        "policy": "min_peak_then_time_within_relative_update_tolerance",
        "relative_time_tolerance": relative_time_tolerance,
        "original_predicted_update_ms": ms0, "selected_predicted_update_ms": best[1],
        "original_peak_bytes": peak0, "selected_peak_bytes": best[0],
        "original_microbatches": len(plan.microbatches), "selected_microbatches": len(selected.microbatches),
        "candidates_examined": examined, "changed": selected != plan, "repacked_families": changes,
        "scope": "bounded homogeneous rank-resident CP1 repacking; distributed batches unchanged",
        "global_optimality_certificate": False}
