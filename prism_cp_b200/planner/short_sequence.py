"""Short-sequence refinement: split CP groups inside their parent rank domains.

Keeps microbatch rounds and parent rank domains; redistributes whole samples
of a group over child groups of smaller CP (CP1 preferred, recursively mixed
CP1/2/4), accepting a change only if the complete-plan objective strictly
improves and the number of executed (coalesced) microbatches does not grow.
Ties preserve the input plan. Rules as the reference's
(experiments/sequence_dynamic_cp/short_sequence.py:15-153).
"""

from __future__ import annotations

import math
import time

from .mixed import coalesce_rounds
from .onedim import Group, _fits, validate


def refine_short_sequences(plan, lengths, limits, cost) -> dict:
    started = time.perf_counter()
    validate(plan, lengths, limits)
    windows = coalesce_rounds(plan, lengths, limits.world, limits.token_cap, limits.max_sequences)
    window_of = {i: w for w, rows in enumerate(windows) for i in rows}
    tokens = [[0] * limits.world for _ in windows]
    counts = [[0] * limits.world for _ in windows]
    for i, row in enumerate(plan):
        for g in row:
            for r in g.ranks:
                tokens[window_of[i]][r] += sum(lengths[k] for k in g.ids) // len(g.ranks)
                counts[window_of[i]][r] += len(g.ids)
    times: dict = {}
    weights: dict = {}
    memo: dict = {}
    attempted = 0
    proxy = getattr(cost, "seed_proxy", cost)

    def elapsed(g):
        if g not in times:
            v = float(cost.group(g, lengths)["cost"])
            if not math.isfinite(v) or v < 0:
                raise ValueError("Invalid short-sequence group cost")
            times[g] = v
        return times[g]

    def preference(groups):
        short = [(sum(lengths[i] for i in g.ids if lengths[i] <= limits.token_cap), len(g.ranks)) for g in groups]
        return (sum(n for n, cp in short if cp > 1), sum(n * (cp - 1) for n, cp in short),
                max(elapsed(g) for g in groups),
                sum(sum(lengths[i] for i in g.ids) * (len(g.ranks) - 1) for g in groups))

    def partition(parent, cp, placement):
        ranks = [parent.ranks[j:j + cp] for j in range(0, len(parent.ranks), cp)]
        if len(parent.ids) < len(ranks) or max(lengths[i] for i in parent.ids) > cp * limits.token_cap:
            return None
        bins = [[] for _ in ranks]
        loads, work = [0] * len(ranks), [0.0] * len(ranks)
        for i in sorted(parent.ids, key=lambda k: (-lengths[k], k)):
            if i not in weights:
                weights[i] = proxy.group(Group((parent.ranks[0],), (i,)), lengths)["cost"]
            opts = [j for j in range(len(ranks)) if loads[j] + lengths[i] <= cp * limits.token_cap
                    and (limits.max_sequences is None or len(bins[j]) < limits.max_sequences)]
            if not opts:
                return None
            empty = [j for j in opts if not bins[j]]
            if empty:
                opts = empty  # every child must get a sample
            if placement == "balanced":
                j = min(opts, key=lambda j: (work[j], loads[j], j))
            else:
                j = min(opts, key=lambda j: (-loads[j], work[j], j))
            bins[j].append(i)
            loads[j] += lengths[i]
            work[j] += weights[i]
        order = {i: j for j, i in enumerate(parent.ids)}
        groups = tuple(Group(r, tuple(sorted(ids, key=order.__getitem__))) for r, ids in zip(ranks, bins))
        if any(not _fits(g.ids, cp, lengths, limits)
               or (hasattr(cost, "feasible_group") and not cost.feasible_group(g.ids, cp, lengths))
               for g in groups):
            return None
        return groups

    def refine(parent):
        nonlocal attempted
        if parent in memo:
            return memo[parent]
        best = (parent,)
        before = elapsed(parent)
        cp = limits.min_cp
        while cp < len(parent.ranks):
            tried = set()
            for placement in ("balanced", "best_fit"):
                children = partition(parent, cp, placement)
                if children is None or children in tried:
                    continue
                tried.add(children)
                attempted += 1
                candidate = tuple(g for child in children for g in refine(child))
                after = max(elapsed(g) for g in candidate)
                if after <= before + 1e-9 * max(1.0, abs(before)) and preference(candidate) < preference(best):
                    best = candidate
            cp *= 2
        memo[parent] = best
        return best

    result, split_groups, rejected_windows = [], 0, 0
    for i, row in enumerate(plan):
        new_row = []
        w = window_of[i]
        for parent in row:
            children = refine(parent)
            old = sum(lengths[k] for k in parent.ids) // len(parent.ranks)
            delta = [(r, sum(lengths[k] for k in g.ids) // len(g.ranks) - old, len(g.ids) - len(parent.ids))
                     for g in children for r in g.ranks]
            fits = all(tokens[w][r] + dt <= limits.token_cap
                       and (limits.max_sequences is None or counts[w][r] + dc <= limits.max_sequences)
                       for r, dt, dc in delta)
            if not fits:
                rejected_windows += 1
                children = (parent,)
            else:
                for r, dt, dc in delta:
                    tokens[w][r] += dt
                    counts[w][r] += dc
            split_groups += children != (parent,)
            new_row.extend(children)
        result.append(tuple(new_row))
    result = tuple(result)
    validate(result, lengths, limits)
    before, after = cost.evaluate(plan, lengths), cost.evaluate(result, lengths)
    tol = 1e-9 * max(1.0, abs(before))
    if after > before + tol:
        raise ValueError("Short-sequence refinement increased the complete-plan objective")
    execution = coalesce_rounds(result, lengths, limits.world, limits.token_cap, limits.max_sequences)
    if len(execution) > len(windows):
        raise ValueError("Short-sequence refinement increased execution microbatches")
    cand_score, cand_splits = after, split_groups
    tie = result != plan and not after < before - tol
    if tie:
        result, after, split_groups, execution = plan, before, 0, windows
    return {"plan": result, "score_before": before, "score_after": after, "split_groups": split_groups,
            "partition_candidates": attempted, "candidate_score_after": cand_score,
            "candidate_split_groups": cand_splits, "rejected_objective_tie": tie,
            "rejected_execution_windows": rejected_windows, "execution_microbatches_before": len(windows),
            "execution_microbatches_after": len(execution),
            "planning_ms": (time.perf_counter() - started) * 1000,
            "scope": "strict complete source-objective improvement; ties preserve input plan; preserve "
                     "mixed-window feasibility; no GPU timing or memory model"}
