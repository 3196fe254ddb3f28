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


def round_load(groups, lengths, world: int) -> tuple[list[int], list[int]]:
    """Per-rank (tokens, packed sequences) one scheduling round puts on every rank."""
    tokens, seqs = [0] * world, [0] * world
    for g in groups:
        share, rest = divmod(sum(lengths[i] for i in g.ids), len(g.ranks))
        if rest:
            raise ValueError("CP token count is not integral")
        for r in g.ranks:
            tokens[r] += share
            seqs[r] += len(g.ids)
    return tokens, seqs


class _Window:
    """Rounds merged into one microbatch so far, with their per-rank totals."""

    def __init__(self, world: int):
        self.rounds: list[int] = []
        self.tokens, self.seqs = [0] * world, [0] * world

    def admits(self, tokens, seqs, token_cap: int, max_sequences) -> bool:
        if any(a + b > token_cap for a, b in zip(self.tokens, tokens)):
            return False
        return max_sequences is None or all(a + b <= max_sequences for a, b in zip(self.seqs, seqs))

    def take(self, ordinal: int, tokens, seqs) -> None:
        self.rounds.append(ordinal)
        self.tokens = [a + b for a, b in zip(self.tokens, tokens)]
        self.seqs = [a + b for a, b in zip(self.seqs, seqs)]


def coalesce_rounds(plan, lengths, world, token_cap, max_sequences=None):
    """Consecutive rounds of a 1-D plan merged greedily into windows (tuples of round
    indices) whose per-rank token and sequence totals stay within the caps."""
    windows, window = [], _Window(world)
    for ordinal, groups in enumerate(plan):
        tokens, seqs = round_load(groups, lengths, world)
        if max(tokens) > token_cap:
            raise ValueError("Original round exceeds token capacity")
        if window.rounds and not window.admits(tokens, seqs, token_cap, max_sequences):
            windows.append(tuple(window.rounds))
            window = _Window(world)
        window.take(ordinal, tokens, seqs)
    if window.rounds:
        windows.append(tuple(window.rounds))
    return tuple(windows)


def local_execution_groups(state: dict, ordinal: int, rank: int):
    """The groups ``rank`` runs in execution window ``ordinal`` (one per merged round)."""
    windows = state.get("execution_rounds")
    members = (ordinal,) if windows is None else windows[ordinal]
    picked = []
    for i in members:
        picked.append(next(g for g in state["plan"][i] if rank in g.ranks))
    return tuple(picked)


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
        conflict = False
        owner: dict[int, tuple] = {}
        for i in window:
            for g in plan[i]:
                for r in g.ranks:
                    if owner.setdefault(r, g.ranks) != g.ranks:
                        conflict = True
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
