"""Immutable token-ownership IR of a joint (sequence x layer) CP plan.

A token is identified by ``(sample, position)``. A ``Layout`` assigns every
sample of a microbatch to one CP group (an aligned dyadic rank interval) and a
partition mode: ``zigzag`` (GQA: each sample cut into 2*cp chunks, rank i holds
chunks i and 2cp-1-i) or ``contiguous`` (GDN: the group's packed samples sliced
evenly). A ``Microbatch`` has an ingress layout and one ``(attention, mlp)``
layout pair per transformer layer; a ``Plan`` is a world size, a layer pattern
over ``{G, *}`` and the microbatches. JSON schema name: ``joint_cp_v1``.

Behavioural parity with the reference IR
(experiments/sequence_dynamic_cp/joint_cp/ir.py:11-166): the same dataclass
fields, the same validation rules and messages' intent, the same span and
route semantics (edges ``(src, dst, src_offset, dst_offset, count)``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable

SCHEMA = "joint_cp_v1"
MODES = ("zigzag", "contiguous")


@dataclass(frozen=True, order=True)
class Group:
    ranks: tuple[int, ...]
    samples: tuple[int, ...]


@dataclass(frozen=True)
class Layout:
    groups: tuple[Group, ...]
    mode: str

    def with_mode(self, mode: str) -> "Layout":
        return Layout(self.groups, mode)

    def sample_cp(self) -> tuple[tuple[int, int], ...]:
        return tuple(sorted((s, len(g.ranks)) for g in self.groups for s in g.samples))

    def tokens(self, lengths, world: int) -> tuple[int, ...]:
        per_rank = [0] * world
        for g in self.groups:
            share = sum(lengths[s] for s in g.samples) // len(g.ranks)
            for r in g.ranks:
                per_rank[r] = share
        return tuple(per_rank)

    def rank_ids(self, world: int) -> list[list[int]]:
        out: list[list[int]] = [[] for _ in range(world)]
        for g in self.groups:
            for r in g.ranks:
                out[r] = list(g.samples)
        return out

    def group_of(self, rank: int) -> Group:
        for g in self.groups:
            if rank in g.ranks:
                return g
        raise KeyError(rank)


@dataclass(frozen=True)
class Microbatch:
    ingress: Layout
    layers: tuple[tuple[Layout, Layout], ...]   # (attention, mlp) per layer


@dataclass(frozen=True)
class Plan:
    world: int
    pattern: str
    microbatches: tuple[Microbatch, ...]

    def to_dict(self) -> dict:
        def lay(x: Layout):
            return {"groups": [{"ranks": list(g.ranks), "samples": list(g.samples)} for g in x.groups],
                    "mode": x.mode}
        return {"schema": SCHEMA, "world": self.world, "pattern": self.pattern,
                "microbatches": [{"ingress": lay(b.ingress), "layers": [[lay(a), lay(m)] for a, m in b.layers]}
                                 for b in self.microbatches]}

    @classmethod
    def from_dict(cls, data: dict) -> "Plan":
        if data.get("schema") != SCHEMA:
            raise ValueError("Unknown joint plan schema")

        def lay(row) -> Layout:
            return Layout(tuple(Group(tuple(g["ranks"]), tuple(g["samples"])) for g in row["groups"]), row["mode"])

        return cls(int(data["world"]), str(data["pattern"]),
                   tuple(Microbatch(lay(b["ingress"]), tuple((lay(a), lay(m)) for a, m in b["layers"]))
                         for b in data["microbatches"]))


def is_dyadic_interval(ranks: tuple[int, ...]) -> bool:
    cp = len(ranks)
    return (cp > 0 and cp & (cp - 1) == 0 and ranks[0] % cp == 0
            and ranks == tuple(range(ranks[0], ranks[0] + cp)))


def validate_layout(layout: Layout, lengths, world: int) -> frozenset:
    if layout.mode not in MODES:
        raise ValueError("Unknown ownership mode")
    covered_ranks: list[int] = []
    seen: list[int] = []
    for g in layout.groups:
        cp = len(g.ranks)
        if not is_dyadic_interval(g.ranks):
            raise ValueError("CP groups must be aligned dyadic rank intervals")
        if not g.samples:
            raise ValueError("Every executing group must have nonempty work")
        for s in g.samples:
            if s not in lengths or type(lengths[s]) is not int or lengths[s] <= 0:
                raise ValueError("Unknown sample or invalid length")
            if cp > 1 and lengths[s] % (2 * cp):
                raise ValueError("Unpadded backend requires sequence alignment to 2*CP")
        covered_ranks.extend(g.ranks)
        seen.extend(g.samples)
    if sorted(covered_ranks) != list(range(world)):
        raise ValueError("Each rank must execute exactly one group per layer")
    if len(seen) != len(set(seen)):
        raise ValueError("Layout duplicates a sample")
    return frozenset(seen)


def validate_plan(plan: Plan, lengths) -> None:
    w = plan.world
    if not w or w & (w - 1):
        raise ValueError("World must be a positive power of two")
    if not plan.pattern or set(plan.pattern) - set("G*"):
        raise ValueError("Pattern must contain GDN G and/or GQA *")
    covered: set = set()
    for mb in plan.microbatches:
        ids = validate_layout(mb.ingress, lengths, w)
        if mb.ingress.mode != "zigzag" or len(mb.layers) != len(plan.pattern):
            raise ValueError("Invalid ingress or layer count")
        if covered & ids:
            raise ValueError("Microbatches duplicate samples")
        covered |= ids
        for symbol, (attention, mlp) in zip(plan.pattern, mb.layers):
            want = "contiguous" if symbol == "G" else "zigzag"
            if attention.mode != want:
                raise ValueError("Attention ownership mode disagrees with kernel")
            for lay in (attention, mlp):
                if validate_layout(lay, lengths, w) != ids:
                    raise ValueError("Layer ownership changes the microbatch sample set")
    if covered != set(lengths):
        raise ValueError("Plan does not cover the complete input exactly once")


Span = tuple[int, int, int, int]   # (sample, logical start, local offset, count)


def spans(layout: Layout, lengths, world: int) -> tuple[tuple[Span, ...], ...]:
    """Per-rank token intervals in local order, without materialising tokens."""
    rows: list[list[Span]] = [[] for _ in range(world)]
    for g in layout.groups:
        cp = len(g.ranks)
        width = sum(lengths[s] for s in g.samples) // cp
        for index, rank in enumerate(g.ranks):
            local = 0
            packed = 0
            for s in g.samples:
                n = lengths[s]
                if layout.mode == "zigzag":
                    if cp == 1:
                        pieces = [(0, n)]
                    else:
                        c = n // (2 * cp)
                        pieces = [(index * c, c), ((2 * cp - 1 - index) * c, c)]
                else:
                    lo = max(packed, index * width)
                    hi = min(packed + n, (index + 1) * width)
                    pieces = [(lo - packed, hi - lo)] if hi > lo else []
                for begin, count in pieces:
                    rows[rank].append((s, begin, local, count))
                    local += count
                packed += n
    return tuple(tuple(r) for r in rows)


Edge = tuple[int, int, int, int, int]  # (src rank, dst rank, src offset, dst offset, count)


def route(source: Layout, target: Layout, lengths, world: int) -> tuple[Edge, ...]:
    """Exact permutation edges moving every token from ``source`` to ``target``."""
    if validate_layout(source, lengths, world) != validate_layout(target, lengths, world):
        raise ValueError("Routing requires identical sample sets")
    src_rows, dst_rows = spans(source, lengths, world), spans(target, lengths, world)
    owners: dict[int, list[tuple[int, int, int, int]]] = {}
    for rank, row in enumerate(dst_rows):
        for s, begin, off, count in row:
            owners.setdefault(s, []).append((rank, begin, off, count))
    edges = []
    for rank, row in enumerate(src_rows):
        for s, begin, off, count in row:
            for other, obegin, ooff, ocount in owners[s]:
                lo, hi = max(begin, obegin), min(begin + count, obegin + ocount)
                if hi > lo:
                    edges.append((rank, other, off + lo - begin, ooff + lo - obegin, hi - lo))
    return tuple(sorted(edges))


def identity_route(edges: Iterable[Edge]) -> bool:
    return all(s == d and a == b for s, d, a, b, _ in edges)
