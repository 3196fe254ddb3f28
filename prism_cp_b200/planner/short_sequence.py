"""Short-sequence refinement: split CP groups inside their parent rank domains.

A CP group's ranks may run its samples better as several smaller groups (CP1
preferred): whole samples are redistributed over child groups that partition
the parent's ranks, recursively, so a CP4 group can become CP2 + CP1 + CP1.
Rounds and parent rank domains never change. A split is kept only if

* the split group is no slower than the parent under the cost model,
* it moves more of the short (<= K tokens) samples to CP1 (then less
  replication, then a faster critical group, then less total replication),
* every rank of the execution window still fits its token / sequence caps,

and the refined plan as a whole must strictly improve the objective without
adding execution microbatches; a tie keeps the input plan. Rules and outputs as
the reference's short_sequence.py:15-153.

Structure: ``_Splitter`` owns the caches and the recursive search of one plan;
``_WindowBudget`` tracks per-window, per-rank headroom while splits are applied.
"""

from __future__ import annotations

import math
import time

from .mixed import coalesce_rounds, round_load
from .onedim import Group, group_fits, validate


class _Splitter:
    PLACEMENTS = ("balanced", "best_fit")

    def __init__(self, lengths, limits, cost):
        self.lengths, self.limits, self.cost = lengths, limits, cost
        self.proxy = getattr(cost, "seed_proxy", cost)
        self.group_ms: dict = {}
        self.sample_work: dict = {}
        self.best: dict = {}
        self.attempted = 0

    def ms(self, g: Group) -> float:
        if g not in self.group_ms:
            value = float(self.cost.group(g, self.lengths)["cost"])
            if not (math.isfinite(value) and value >= 0):
                raise ValueError("Invalid short-sequence group cost")
            self.group_ms[g] = value
        return self.group_ms[g]

    def rank(self, groups) -> tuple:
        """Lower is better: short tokens left on CP > 1, their replication, the critical group's
        time, total replication."""
        cap = self.limits.token_cap
        short_multi = short_repl = total_repl = 0
        for g in groups:
            cp = len(g.ranks)
            short = sum(self.lengths[i] for i in g.ids if self.lengths[i] <= cap)
            if cp > 1:
                short_multi += short
            short_repl += short * (cp - 1)
            total_repl += sum(self.lengths[i] for i in g.ids) * (cp - 1)
        return short_multi, short_repl, max(self.ms(g) for g in groups), total_repl

    def _work(self, parent: Group, i: int) -> float:
        if i not in self.sample_work:
            self.sample_work[i] = self.proxy.group(Group((parent.ranks[0],), (i,)), self.lengths)["cost"]
        return self.sample_work[i]

    def split(self, parent: Group, cp: int, placement: str):
        """Whole samples of ``parent`` packed onto its rank blocks of size ``cp``, largest first
        (each block gets a sample before any block gets a second); None if infeasible."""
        lim, L = self.limits, self.lengths
        blocks = [parent.ranks[j:j + cp] for j in range(0, len(parent.ranks), cp)]
        room = cp * lim.token_cap
        if len(parent.ids) < len(blocks) or max(L[i] for i in parent.ids) > room:
            return None
        bins = [[] for _ in blocks]
        load = [0] * len(blocks)
        work = [0.0] * len(blocks)
        for i in sorted(parent.ids, key=lambda k: (-L[k], k)):
            w = self._work(parent, i)
            open_ = [j for j in range(len(blocks)) if load[j] + L[i] <= room
                     and (lim.max_sequences is None or len(bins[j]) < lim.max_sequences)]
            if not open_:
                return None
            empty = [j for j in open_ if not bins[j]]
            pool = empty or open_
            if placement == "balanced":
                j = min(pool, key=lambda j: (work[j], load[j], j))
            else:
                j = min(pool, key=lambda j: (-load[j], work[j], j))
            bins[j].append(i)
            load[j] += L[i]
            work[j] += w
        position = {i: p for p, i in enumerate(parent.ids)}
        children = tuple(Group(b, tuple(sorted(ids, key=position.__getitem__))) for b, ids in zip(blocks, bins))
        feasible = getattr(self.cost, "feasible_group", None)
        for g in children:
            if not group_fits(g.ids, cp, L, lim) or (feasible is not None and not feasible(g.ids, cp, L)):
                return None
        return children

    def refine(self, parent: Group) -> tuple:
        """The best split of ``parent`` (itself when nothing beats it), memoised."""
        if parent in self.best:
            return self.best[parent]
        chosen, limit = (parent,), self.ms(parent)
        limit += 1e-9 * max(1.0, abs(limit))
        cp = self.limits.min_cp
        while cp < len(parent.ranks):
            tried = set()
            for placement in self.PLACEMENTS:
                children = self.split(parent, cp, placement)
                if children is None or children in tried:
                    continue
                tried.add(children)
                self.attempted += 1
                flat = tuple(g for child in children for g in self.refine(child))
                if max(self.ms(g) for g in flat) <= limit and self.rank(flat) < self.rank(chosen):
                    chosen = flat
            cp *= 2
        self.best[parent] = chosen
        return chosen


class _WindowBudget:
    """Per execution window and rank: tokens and packed sequences placed so far."""

    def __init__(self, plan, lengths, limits, windows):
        self.lengths, self.limits = lengths, limits
        self.window_of = {r: w for w, rounds in enumerate(windows) for r in rounds}
        self.tokens = [[0] * limits.world for _ in windows]
        self.seqs = [[0] * limits.world for _ in windows]
        for r, row in enumerate(plan):
            t, s = round_load(row, lengths, limits.world)
            w = self.window_of[r]
            self.tokens[w] = [a + b for a, b in zip(self.tokens[w], t)]
            self.seqs[w] = [a + b for a, b in zip(self.seqs[w], s)]

    def _share(self, g: Group) -> int:
        return sum(self.lengths[k] for k in g.ids) // len(g.ranks)

    def apply(self, round_index: int, parent: Group, children: tuple) -> bool:
        """Book replacing ``parent`` by ``children`` if every rank still fits; False otherwise."""
        w, lim = self.window_of[round_index], self.limits
        base_tokens, base_seqs = self._share(parent), len(parent.ids)
        delta = [(r, self._share(g) - base_tokens, len(g.ids) - base_seqs) for g in children for r in g.ranks]
        for r, dt, ds in delta:
            if self.tokens[w][r] + dt > lim.token_cap:
                return False
            if lim.max_sequences is not None and self.seqs[w][r] + ds > lim.max_sequences:
                return False
        for r, dt, ds in delta:
            self.tokens[w][r] += dt
            self.seqs[w][r] += ds
        return True


def refine_short_sequences(plan, lengths, limits, cost) -> dict:
    started = time.perf_counter()
    validate(plan, lengths, limits)
    windows = coalesce_rounds(plan, lengths, limits.world, limits.token_cap, limits.max_sequences)
    splitter = _Splitter(lengths, limits, cost)
    budget = _WindowBudget(plan, lengths, limits, windows)
    rows, splits, rejected = [], 0, 0
    for r, row in enumerate(plan):
        out = []
        for parent in row:
            children = splitter.refine(parent)
            if not budget.apply(r, parent, children):
                rejected += 1
                children = (parent,)
            splits += children != (parent,)
            out.extend(children)
        rows.append(tuple(out))
    refined = tuple(rows)
    validate(refined, lengths, limits)
    before, after = cost.evaluate(plan, lengths), cost.evaluate(refined, lengths)
    tol = 1e-9 * max(1.0, abs(before))
    if after > before + tol:
        raise ValueError("Short-sequence refinement increased the complete-plan objective")
    execution = coalesce_rounds(refined, lengths, limits.world, limits.token_cap, limits.max_sequences)
    if len(execution) > len(windows):
        raise ValueError("Short-sequence refinement increased execution microbatches")
    candidate_after, candidate_splits = after, splits
    # a split whose saving hides behind another group's critical path is a tie: keep the input
    tie = refined != plan and not after < before - tol
    if tie:
        refined, after, splits, execution = plan, before, 0, windows
    return {"plan": refined, "score_before": before, "score_after": after, "split_groups": splits,
            "partition_candidates": splitter.attempted, "candidate_score_after": candidate_after,
            "candidate_split_groups": candidate_splits, "rejected_objective_tie": tie,
            "rejected_execution_windows": rejected, "execution_microbatches_before": len(windows),
            "execution_microbatches_after": len(execution),
            "planning_ms": (time.perf_counter() - started) * 1000,
            "scope": "strict complete source-objective improvement; ties preserve input plan; preserve "
                     "mixed-window feasibility; no GPU timing or memory model"}
