"""Mixed-CP execution: coalesce consecutive scheduling rounds into one microbatch.

Rounds (groups of a 1-D plan) are merged in order while every rank's token sum
stays <= the per-rank cap (and the packed-sequence cap). CP segments of
different sizes then run in one microbatch: tokenwise GEMMs over all segments
once, attention / GDN per segment with its own team (reference:
experiments/sequence_dynamic_cp/mixed_plan.py:8-38). ``to_joint`` expresses a
coalesced window as a joint-IR microbatch the executor runs directly.
"""

from __future__ import annotations

from .joint.ir import Group as JGroup, Layout, Microbatch, Plan as JointPlan


def coalesce_rounds(plan, lengths, world, token_cap, max_sequences=None):
    batches, current = [], []
    tokens, counts = [0] * world, [0] * world
    for ordinal, groups in enumerate(plan):
        added, seqs = [0] * world, [0] * world
        for g in groups:
            total = sum(lengths[i] for i in g.ids)
            if total % len(g.ranks):
                raise ValueError("CP token count is not integral")
            for r in g.ranks:
                added[r] += total // len(g.ranks)
                seqs[r] += len(g.ids)
        if any(n > token_cap for n in added):
            raise ValueError("Original round exceeds token capacity")
        over = any(a + b > token_cap for a, b in zip(tokens, added)) or (
            max_sequences is not None and any(a + b > max_sequences for a, b in zip(counts, seqs)))
        if current and over:
            batches.append(tuple(current))
            current, tokens, counts = [], [0] * world, [0] * world
        current.append(ordinal)
        tokens = [a + b for a, b in zip(tokens, added)]
        counts = [a + b for a, b in zip(counts, seqs)]
    if current:
        batches.append(tuple(current))
    return tuple(batches)


def local_execution_groups(state: dict, ordinal: int, rank: int):
    rounds = state.get("execution_rounds")
    indices = rounds[ordinal] if rounds is not None else (ordinal,)
    return tuple(next(g for g in state["plan"][i] if rank in g.ranks) for i in indices)


def to_joint(plan, lengths, world: int, pattern: str, token_cap: int | None = None,
             max_sequences: int | None = None) -> JointPlan:
    """A 1-D plan as a joint plan (one layout per microbatch, kernel modes per layer).

    Without ``token_cap`` every round is its own microbatch. With it, rounds are
    coalesced and a window whose rounds use different teams on one rank is split
    back into rounds (a rank runs one team per layer in the joint IR).
    """
    windows = (coalesce_rounds(plan, lengths, world, token_cap, max_sequences) if token_cap
               else tuple((i,) for i in range(len(plan))))
    mbs = []
    for window in windows:
        merged: dict[tuple, list[int]] = {}
        conflict = False
        owner: dict[int, tuple] = {}
        for i in window:
            for g in plan[i]:
                for r in g.ranks:
                    if r in owner and owner[r] != g.ranks:
                        conflict = True
                    owner[r] = g.ranks
                merged.setdefault(g.ranks, []).extend(g.ids)
        parts = [[i] for i in window] if conflict else [list(window)]
        for part in parts:
            groups: dict[tuple, list[int]] = {}
            for i in part:
                for g in plan[i]:
                    groups.setdefault(g.ranks, []).extend(g.ids)
            jg = tuple(JGroup(r, tuple(ids)) for r, ids in sorted(groups.items()))
            zig, cont = Layout(jg, "zigzag"), Layout(jg, "contiguous")
            mbs.append(Microbatch(zig, tuple((cont, cont) if c == "G" else (zig, zig) for c in pattern)))
    return JointPlan(world, pattern, tuple(mbs))
