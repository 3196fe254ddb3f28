"""One-dimensional CP planner: one set of CP groups for every layer of a microbatch.

API (same names and semantics as the reference's planner,
experiments/sequence_dynamic_cp/planner.py:18-475):

* ``Constraints(world, token_cap, min_cp, max_sequences, alignment)``
* ``Group(ranks, ids)``; a plan is a tuple of microbatches, each a tuple of groups
* ``from_rank_ids`` / ``to_rank_ids``: the executor's replicated sample-id codec
* ``validate``: aligned dyadic groups, capacity, exactly-once coverage
* ``ProxyCost(a, b)``: ``a * Q + b * L`` per group (Q in Ki^2/cp, L in Ki/cp);
  ``beta_tokens = b / a * 1024`` is the weighted-native ablation
* ``ExactCosts``: measured complete-plan table keyed by ``fingerprint``
* ``native_plan``, ``pack_layout`` (LPT into a fixed CP-size vector), ``layouts``
  (homogeneous + dyadic neighbours of native), local move/swap ``search`` with the
  short-sequence refinement pass, ``select`` (measured > proxy opt-in > native),
  ``export_plan`` and ``models`` (CP1 stack coefficients).
"""

from __future__ import annotations

import json
import math
import time
from dataclasses import dataclass
from pathlib import Path

from .inputs import fingerprint as _fingerprint
from .native import replay


@dataclass(frozen=True)
class Group:
    ranks: tuple[int, ...]
    ids: tuple[int, ...]


Plan = tuple  # tuple[tuple[Group, ...], ...]


@dataclass(frozen=True)
class Constraints:
    world: int
    token_cap: int
    min_cp: int = 1
    max_sequences: int | None = None
    alignment: int = 1

    def __post_init__(self):
        for v in (self.world, self.min_cp):
            if v < 1 or v & (v - 1):
                raise ValueError("First version requires power-of-two world and min_cp")
        if self.min_cp > self.world or self.token_cap < 1 or self.alignment < 1:
            raise ValueError("Invalid CP/token/alignment constraint")
        if self.max_sequences is not None and self.max_sequences < 1:
            raise ValueError("max_sequences must be positive")


def from_rank_ids(batches) -> Plan:
    out = []
    for batch in batches:
        owners: dict[tuple, list[int]] = {}
        for rank, ids in enumerate(batch):
            owners.setdefault(tuple(ids), []).append(rank)
        out.append(tuple(Group(tuple(r), ids) for ids, r in owners.items()))
    return tuple(out)


def to_rank_ids(plan: Plan, world: int):
    out = []
    for batch in plan:
        ranks: list[list[int]] = [[] for _ in range(world)]
        for g in batch:
            for r in g.ranks:
                ranks[r] = list(g.ids)
        out.append(ranks)
    return out


def validate(plan: Plan, lengths: dict, limits: Constraints) -> None:
    if any(not isinstance(i, int) or not isinstance(n, int) or n <= 0 or n % limits.alignment
           for i, n in lengths.items()):
        raise ValueError("IDs/lengths must be integers; lengths must be positive and aligned")
    if not plan or not lengths:
        raise ValueError("Empty steps are unsupported")
    seen = []
    for batch in plan:
        ranks = []
        for g in batch:
            cp = len(g.ranks)
            if not cp or cp & (cp - 1) or cp < limits.min_cp or not g.ids:
                raise ValueError("Empty or unsupported CP group")
            if g.ranks[0] % cp or g.ranks != tuple(range(g.ranks[0], g.ranks[0] + cp)):
                raise ValueError("CP group must match a precreated aligned contiguous group")
            if any(i not in lengths for i in g.ids):
                raise ValueError("Unknown sample ID")
            if cp > 1 and any(lengths[i] % (2 * cp) for i in g.ids):
                raise ValueError("THD zigzag requires sequence padding divisible by 2*CP")
            if sum(lengths[i] for i in g.ids) > limits.token_cap * cp:
                raise ValueError("Per-rank token capacity exceeded")
            if limits.max_sequences is not None and len(g.ids) > limits.max_sequences:
                raise ValueError("Real packed-sequence capacity exceeded")
            ranks.extend(g.ranks)
            seen.extend(g.ids)
        if sorted(ranks) != list(range(limits.world)):
            raise ValueError("All ranks must execute exactly one nonempty group per microbatch")
    if sorted(seen) != sorted(lengths):
        raise ValueError("Samples must appear exactly once at group level across the full step")


@dataclass(frozen=True)
class ProxyCost:
    name: str
    a: float
    b: float
    provenance: str = "conditional_CP1_compute_divided_by_CP"

    def __post_init__(self):
        if not all(math.isfinite(v) and v >= 0 for v in (self.a, self.b)) or self.a + self.b == 0:
            raise ValueError("Cost coefficients must be finite, nonnegative and nonzero")

    @property
    def beta_tokens(self) -> float:
        if self.a <= 0:
            raise ValueError("Weighted native ablation requires positive quadratic coefficient")
        return self.b / self.a * 1024

    def group(self, group: Group, lengths: dict) -> dict:
        cp = len(group.ranks)
        q = sum((lengths[i] / 1024) ** 2 for i in group.ids) / cp
        l = sum(lengths[i] / 1024 for i in group.ids) / cp
        return {"q_ki2": q, "l_ki": l, "quadratic": self.a * q, "linear": self.b * l,
                "cost": self.a * q + self.b * l}

    def evaluate(self, plan: Plan, lengths: dict) -> float:
        return sum(max(self.group(g, lengths)["cost"] for g in batch) for batch in plan)


def fingerprint(plan: Plan, lengths: dict) -> str:
    return _fingerprint(plan, lengths)


class ExactCosts:
    """Complete-plan timings frozen for one model/runtime/topology contract."""

    def __init__(self, data: dict, contract: dict):
        if data["contract"] != contract:
            raise ValueError("Measured costs do not match model/backend/topology contract")
        self.scope = data["scope"]
        self.records = {}
        seen = set()
        for row in data["records"]:
            key = row["fingerprint"]
            if key in seen:
                raise ValueError("Duplicate exact-plan measurement")
            seen.add(key)
            if row["status"] == "ok" and row["numerical_pass"] is True:
                v = row["milliseconds"]
                if not math.isfinite(v) or v <= 0:
                    raise ValueError("Invalid complete-plan measurement")
                self.records[key] = row

    def evaluate(self, plan: Plan, lengths: dict):
        row = self.records.get(fingerprint(plan, lengths))
        return row["milliseconds"] if row else None


def native_plan(lengths: dict, limits: Constraints, cost: ProxyCost) -> Plan:
    plan = from_rank_ids(replay(list(lengths.items()), limits.world, limits.token_cap, limits.min_cp,
                                cost.beta_tokens))
    validate(plan, lengths, limits)
    return plan


def _fits(ids, cp, lengths, limits) -> bool:
    return (bool(ids) and sum(lengths[i] for i in ids) <= cp * limits.token_cap
            and (limits.max_sequences is None or len(ids) <= limits.max_sequences)
            and (cp == 1 or all(lengths[i] % (2 * cp) == 0 for i in ids)))


def pack_layout(lengths: dict, limits: Constraints, sizes: tuple[int, ...], cost) -> Plan:
    """LPT-pack the whole step into a fixed CP-size vector; a partial tail is repacked
    on one world-wide group instead of leaving ranks idle."""
    if sum(sizes) != limits.world:
        raise ValueError("Layout must cover the world")
    remaining = sorted(lengths, key=lambda i: (-lengths[i], i))
    out = []
    while remaining:
        groups, start = [], 0
        for cp in sizes:
            groups.append(Group(tuple(range(start, start + cp)), ()))
            start += cp
        costs = [0.0] * len(groups)
        leftovers = []
        for i in remaining:
            options = []
            for j, g in enumerate(groups):
                ids = (*g.ids, i)
                if _fits(ids, len(g.ranks), lengths, limits) and (
                        not hasattr(cost, "feasible_group") or cost.feasible_group(ids, len(g.ranks), lengths)):
                    new = cost.group(Group(g.ranks, ids), lengths)["cost"]
                    worst = max(new, max((v for k, v in enumerate(costs) if k != j), default=0))
                    options.append((worst, costs[j], j, new))
            if not options:
                leftovers.append(i)
                continue
            _, _, j, new = min(options)
            groups[j] = Group(groups[j].ranks, (*groups[j].ids, i))
            costs[j] = new
        if any(not g.ids for g in groups):
            picked, leftovers = [], []
            for i in remaining:
                (picked if _fits((*picked, i), limits.world, lengths, limits) else leftovers).append(i)
            groups = [Group(tuple(range(limits.world)), tuple(picked))]
        if len(leftovers) == len(remaining):
            raise ValueError("No feasible group for the next sequence")
        out.append(tuple(groups))
        remaining = leftovers
    plan = tuple(out)
    validate(plan, lengths, limits)
    return plan


def layouts(limits: Constraints, seeds) -> list[tuple[int, ...]]:
    found = set()
    cp = limits.min_cp
    while cp <= limits.world:
        found.add((cp,) * (limits.world // cp))
        cp *= 2
    for plan in seeds:
        for batch in plan:
            sizes = tuple(len(g.ranks) for g in batch)
            found.add(sizes)
            for j, s in enumerate(sizes):
                if s > limits.min_cp:
                    found.add((*sizes[:j], s // 2, s // 2, *sizes[j + 1:]))
                if j + 1 < len(sizes) and s == sizes[j + 1] and sum(sizes[:j]) % (2 * s) == 0:
                    found.add((*sizes[:j], 2 * s, *sizes[j + 2:]))
    return sorted(found)


def _neighbors(plan: Plan, lengths: dict, limits: Constraints):
    locs = [(m, j) for m, batch in enumerate(plan) for j in range(len(batch))]

    def replace(changes):
        return tuple(tuple(changes.get((m, j), g) for j, g in enumerate(batch)) for m, batch in enumerate(plan))

    for src_loc in locs:
        src = plan[src_loc[0]][src_loc[1]]
        if len(src.ids) < 2:
            continue
        for i in src.ids:
            for dst_loc in locs:
                if dst_loc == src_loc:
                    continue
                dst = plan[dst_loc[0]][dst_loc[1]]
                ids = (*dst.ids, i)
                if _fits(ids, len(dst.ranks), lengths, limits):
                    yield replace({src_loc: Group(src.ranks, tuple(k for k in src.ids if k != i)),
                                   dst_loc: Group(dst.ranks, ids)})
    for x, src_loc in enumerate(locs):
        src = plan[src_loc[0]][src_loc[1]]
        for dst_loc in locs[x + 1:]:
            dst = plan[dst_loc[0]][dst_loc[1]]
            for i in src.ids:
                for k in dst.ids:
                    if lengths[i] == lengths[k]:
                        continue
                    a = tuple(k if n == i else n for n in src.ids)
                    b = tuple(i if n == k else n for n in dst.ids)
                    if _fits(a, len(src.ranks), lengths, limits) and _fits(b, len(dst.ranks), lengths, limits):
                        yield replace({src_loc: Group(src.ranks, a), dst_loc: Group(dst.ranks, b)})


def search(lengths: dict, limits: Constraints, cost, local_evaluations: int = 128, rounds: int = 2) -> dict:
    """Finite legal candidates (native seeds, layout packings, local moves/swaps,
    short-sequence split). A deterministic evaluation budget, not wall time, so
    every rank computes the same schedule."""
    started = time.perf_counter()
    if local_evaluations < 0 or rounds < 0:
        raise ValueError("Search budgets must be nonnegative")
    candidates: dict[str, dict] = {}
    failures = []

    def add(name, plan):
        validate(plan, lengths, limits)
        key = fingerprint(plan, lengths)
        if key not in candidates:
            candidates[key] = {"name": name, "plan": plan, "proxy_cost": cost.evaluate(plan, lengths),
                               "fingerprint": key}

    seeds = []
    for name, model in (("native_square", ProxyCost("square", 1, 0)),
                        ("native_weighted", getattr(cost, "seed_proxy", cost))):
        try:
            plan = native_plan(lengths, limits, model)
            seeds.append(plan)
            add(name, plan)
        except (ValueError, AssertionError) as error:
            failures.append({"candidate": name, "reason": str(error)})
    for sizes in layouts(limits, seeds):
        try:
            add("layout_" + "x".join(map(str, sizes)), pack_layout(lengths, limits, sizes, cost))
        except ValueError as error:
            failures.append({"candidate": str(sizes), "reason": str(error)})
    if not candidates:
        raise ValueError("No legal candidate for this complete step")

    def better(v, cur):
        return v < cur - 1e-9 * max(1.0, abs(cur))

    best = next(iter(candidates.values()))
    for c in candidates.values():
        if better(c["proxy_cost"], best["proxy_cost"]):
            best = c
    used = 0
    for _ in range(rounds):
        prev = best
        for plan in _neighbors(prev["plan"], lengths, limits):
            if used >= local_evaluations:
                break
            used += 1
            try:
                add("local_move_or_swap", plan)
            except ValueError as error:
                failures.append({"candidate": "local_move_or_swap", "reason": str(error)})
                continue
            v = cost.evaluate(plan, lengths)
            if better(v, best["proxy_cost"]):
                best = candidates[fingerprint(plan, lengths)]
        if best is prev or used >= local_evaluations:
            break
    from .short_sequence import refine_short_sequences
    refinement = refine_short_sequences(best["plan"], lengths, limits, cost)
    if refinement["plan"] != best["plan"]:
        add("short_sequence_split", refinement["plan"])
        best = candidates[fingerprint(refinement["plan"], lengths)]
    return {"selected": best, "candidates": list(candidates.values()), "failures": failures,
            "local_evaluations": used,
            "short_sequence_refinement": {k: v for k, v in refinement.items() if k != "plan"},
            "planning_ms": (time.perf_counter() - started) * 1000, "selection_provenance": cost.provenance,
            "parameter_sync_optimizer": "unknown"}


def select(result: dict, lengths: dict, measured: ExactCosts | None = None, allow_proxy: bool = False):
    native = next((c for c in result["candidates"] if c["name"] == "native_square"), None)
    if measured:
        known = [(measured.evaluate(c["plan"], lengths), j, c) for j, c in enumerate(result["candidates"])]
        known = [(v, j, c) for v, j, c in known if v is not None]
        if known and native and measured.evaluate(native["plan"], lengths) is not None:
            return min(known, key=lambda r: (r[0], r[1]))[2], "measured_complete_plan"
    if allow_proxy:
        return result["selected"], "experimental_compute_proxy"
    if native is None:
        raise ValueError("Native plan is illegal; no calibrated fallback exists")
    return native, "native_fallback_unknown_distributed_cost"


def export_plan(plan: Plan, lengths: dict, cost: ProxyCost, node_size: int) -> dict:
    batches = []
    for batch in plan:
        groups, rq, rl = [], [], []
        for g in batch:
            parts = cost.group(g, lengths)
            rq.extend([parts["q_ki2"]] * len(g.ranks))
            rl.extend([parts["l_ki"]] * len(g.ranks))
            groups.append(dict(ranks=g.ranks, sample_ids=g.ids, padded_lengths=[lengths[i] for i in g.ids],
                               cp=len(g.ranks),
                               placement="intra_node" if len({r // node_size for r in g.ranks}) == 1 else "cross_node",
                               local_tokens=sum(lengths[i] for i in g.ids) / len(g.ranks), **parts))
        batches.append({"groups": groups, "cost": max(g["cost"] for g in groups),
                        "r_q": max(rq) / (sum(rq) / len(rq)), "r_l": max(rl) / (sum(rl) / len(rl))})
    return {"microbatches": batches, "compute_proxy_cost": sum(b["cost"] for b in batches),
            "fingerprint": fingerprint(plan, lengths), "provenance": cost.provenance,
            "memory": "token_cap_only; measured_peak_required", "parameter_sync_optimizer": "unknown"}


def models(path: Path) -> dict[str, ProxyCost]:
    """Proxy models from a CP1 stack-coefficient table (gpt = 4 GQA, hybrid = 1 GQA + 3 GDN)."""
    rows = json.loads(Path(path).read_text())
    chosen = {}
    for name, counts in (("gpt", (4, 0)), ("hybrid", (1, 3))):
        row = next(r for r in rows if (r["gqa_layers"], r["gdn_layers"]) == counts)
        chosen[name] = ProxyCost(name, row["A_ms_per_ki2"], row["B_ms_per_ki"])
    return {"square": ProxyCost("square", 1.0, 0.0, "quadratic_work_proxy_Ki2"), **chosen}
