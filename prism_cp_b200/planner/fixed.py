"""Fixed-CP plans in the joint IR (every layer of a microbatch uses one CP team).

``uniform_plan`` packs samples in order into microbatches of at most
``tokens_per_rank * cp`` tokens and gives each microbatch ``world / cp`` groups
of ``cp`` ranks (samples assigned to the least-loaded group, longest first).
GQA layers use the zigzag mode, GDN layers the contiguous mode, the MLP follows
its attention layout; consecutive GDN/GQA layers therefore reshard at every
GDN<->GQA boundary, as the reference's native N does.
"""

from __future__ import annotations

from .joint.ir import Group, Layout, Microbatch, Plan, validate_plan


def _layers(groups, pattern):
    contiguous = Layout(groups, "contiguous")
    zigzag = Layout(groups, "zigzag")
    return tuple((contiguous, contiguous) if c == "G" else (zigzag, zigzag) for c in pattern)


def microbatch(groups: tuple[Group, ...], pattern: str) -> Microbatch:
    return Microbatch(Layout(groups, "zigzag"), _layers(groups, pattern))


def uniform_plan(lengths: dict[int, int], world: int, cp: int, tokens_per_rank: int, pattern: str) -> Plan:
    if world % cp or cp & (cp - 1):
        raise ValueError("cp must be a power of two dividing the world")
    ngroups = world // cp
    order = sorted(lengths, key=lambda s: (-lengths[s], s))
    cap = tokens_per_rank * cp
    batches = []
    pending = list(order)
    while pending:
        packs = [[] for _ in range(ngroups)]
        loads = [0] * ngroups
        rest = []
        for s in pending:
            j = min(range(ngroups), key=lambda i: (loads[i], i))
            if loads[j] + lengths[s] <= cap or not packs[j]:
                packs[j].append(s)
                loads[j] += lengths[s]
            else:
                rest.append(s)
        if any(not p for p in packs):
            # not enough samples for every group: fall back to one world-wide group
            packs = [sum(packs, [])]
            groups = (Group(tuple(range(world)), tuple(sorted(packs[0]))),)
        else:
            groups = tuple(Group(tuple(range(i * cp, (i + 1) * cp)), tuple(sorted(p))) for i, p in enumerate(packs))
        batches.append(microbatch(groups, pattern))
        pending = rest
    plan = Plan(world, pattern, tuple(batches))
    validate_plan(plan, lengths)
    return plan
