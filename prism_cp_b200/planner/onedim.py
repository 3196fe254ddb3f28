"""One-dimensional CP planner: one set of CP groups for every layer of a microbatch.

A plan is a tuple of microbatches ("rounds"); a microbatch is a tuple of
``Group(ranks, ids)``, each an aligned dyadic rank interval running some whole
samples at CP = len(ranks). The API is the reference planner's
(planner.py:18-475) so its callers and stored plans carry over:

* ``Constraints(world, token_cap, min_cp, max_sequences, alignment)``;
* ``from_rank_ids`` / ``to_rank_ids``: the executor's replicated sample-id codec;
* ``validate``: group legality, per-rank capacity, exactly-once coverage;
* ``ProxyCost(a, b)``: ``a * Q + b * L`` per group (Q in Ki^2 / cp, L in Ki / cp);
  ``beta_tokens = b / a * 1024`` weights the native scheduler's workload;
* ``ExactCosts``: measured complete-plan times keyed by ``fingerprint``;
* ``search``: a finite candidate pool - the native scheduler's plans, an LPT
  packing of every layout in a small family, a budgeted local search of
  sample moves and swaps around the best one, then the short-sequence split;
  ``select`` (measured > proxy opt-in > native) and ``export_plan``.

Design: a ``_Pool`` owns the candidates (deduplicated by fingerprint, first
insertion wins numerical ties); ``_Lpt`` fills one round of a layout;
``neighbours`` enumerates one-step changes of a plan in a fixed order, so the
evaluation budget - not wall time - bounds the search and every rank computes
the same schedule.
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


def _pow2(v: int) -> bool:
    return v >= 1 and v & (v - 1) == 0


@dataclass(frozen=True)
class Constraints:
    world: int
    token_cap: int
    min_cp: int = 1
    max_sequences: int | None = None
    alignment: int = 1

    def __post_init__(self):
        if not (_pow2(self.world) and _pow2(self.min_cp)):
            raise ValueError("First version requires power-of-two world and min_cp")
        if self.min_cp > self.world or min(self.token_cap, self.alignment) < 1:
            raise ValueError("Invalid CP/token/alignment constraint")
        if self.max_sequences is not None and self.max_sequences < 1:
            raise ValueError("max_sequences must be positive")


# ------------------------------------------------------------------ codec
def from_rank_ids(batches) -> Plan:
    """Per-rank sample lists (ranks sharing a list form one group) to a plan."""
    plan = []
    for per_rank in batches:
        teams: dict[tuple, list[int]] = {}
        for rank, ids in enumerate(per_rank):
            teams.setdefault(tuple(ids), []).append(rank)
        plan.append(tuple(Group(tuple(ranks), ids) for ids, ranks in teams.items()))
    return tuple(plan)


def to_rank_ids(plan: Plan, world: int):
    """A plan to per-rank sample lists (every rank of a group lists the group's samples)."""
    out = []
    for batch in plan:
        owner = {r: g.ids for g in batch for r in g.ranks}
        out.append([list(owner.get(r, ())) for r in range(world)])
    return out


# ------------------------------------------------------------------ legality
def _group_problem(g: Group, lengths: dict, limits: Constraints):
    """The first rule ``g`` breaks (as an error message), or None."""
    cp = len(g.ranks)
    if not _pow2(cp) or cp < limits.min_cp or not g.ids:
        return "Empty or unsupported CP group"
    if g.ranks[0] % cp or g.ranks != tuple(range(g.ranks[0], g.ranks[0] + cp)):
        return "CP group must match a precreated aligned contiguous group"
    if not all(i in lengths for i in g.ids):
        return "Unknown sample ID"
    if cp > 1 and any(lengths[i] % (2 * cp) for i in g.ids):
        return "THD zigzag requires sequence padding divisible by 2*CP"
    if sum(lengths[i] for i in g.ids) > limits.token_cap * cp:
        return "Per-rank token capacity exceeded"
    if limits.max_sequences is not None and len(g.ids) > limits.max_sequences:
        return "Real packed-sequence capacity exceeded"
    return None


def validate(plan: Plan, lengths: dict, limits: Constraints) -> None:
    """Raise ValueError unless every microbatch covers every rank with one legal group and
    every sample runs exactly once in the step."""
    for i, n in lengths.items():
        if not isinstance(i, int) or not isinstance(n, int) or n <= 0 or n % limits.alignment:
            raise ValueError("IDs/lengths must be integers; lengths must be positive and aligned")
    if not plan or not lengths:
        raise ValueError("Empty steps are unsupported")
    placed = []
    for batch in plan:
        covered = []
        for g in batch:
            problem = _group_problem(g, lengths, limits)
            if problem:
                raise ValueError(problem)
            covered += g.ranks
            placed += g.ids
        if sorted(covered) != list(range(limits.world)):
            raise ValueError("All ranks must execute exactly one nonempty group per microbatch")
    if sorted(placed) != sorted(lengths):
        raise ValueError("Samples must appear exactly once at group level across the full step")


def group_fits(ids, cp: int, lengths: dict, limits: Constraints) -> bool:
    """Whether samples ``ids`` may form one CP-``cp`` group (capacity, count, zigzag split)."""
    if not ids or sum(lengths[i] for i in ids) > cp * limits.token_cap:
        return False
    if limits.max_sequences is not None and len(ids) > limits.max_sequences:
        return False
    return cp == 1 or all(lengths[i] % (2 * cp) == 0 for i in ids)


# ------------------------------------------------------------------ costs
@dataclass(frozen=True)
class ProxyCost:
    name: str
    a: float
    b: float
    provenance: str = "conditional_CP1_compute_divided_by_CP"

    def __post_init__(self):
        valid = all(math.isfinite(v) and v >= 0 for v in (self.a, self.b))
        if not valid or self.a + self.b == 0:
            raise ValueError("Cost coefficients must be finite, nonnegative and nonzero")

    @property
    def beta_tokens(self) -> float:
        if self.a <= 0:
            raise ValueError("Weighted native ablation requires positive quadratic coefficient")
        return self.b / self.a * 1024

    def group(self, group: Group, lengths: dict) -> dict:
        cp = len(group.ranks)
        ki = [lengths[i] / 1024 for i in group.ids]
        q = sum(x ** 2 for x in ki) / cp
        lin = sum(ki) / cp
        return {"q_ki2": q, "l_ki": lin, "quadratic": self.a * q, "linear": self.b * lin,
                "cost": self.a * q + self.b * lin}

    def evaluate(self, plan: Plan, lengths: dict) -> float:
        """Sum over microbatches of the slowest group's cost."""
        return sum(max(self.group(g, lengths)["cost"] for g in batch) for batch in plan)


def fingerprint(plan: Plan, lengths: dict) -> str:
    return _fingerprint(plan, lengths)


class ExactCosts:
    """Complete-plan timings measured for one model / runtime / topology contract.
    Only rows that ran ("ok") and passed their numerical gate can be selected."""

    def __init__(self, data: dict, contract: dict):
        if data["contract"] != contract:
            raise ValueError("Measured costs do not match model/backend/topology contract")
        self.scope = data["scope"]
        keys = [row["fingerprint"] for row in data["records"]]
        if len(set(keys)) != len(keys):
            raise ValueError("Duplicate exact-plan measurement")
        self.records = {}
        for row in data["records"]:
            if row["status"] != "ok" or row["numerical_pass"] is not True:
                continue
            if not (math.isfinite(row["milliseconds"]) and row["milliseconds"] > 0):
                raise ValueError("Invalid complete-plan measurement")
            self.records[row["fingerprint"]] = row

    def evaluate(self, plan: Plan, lengths: dict):
        row = self.records.get(fingerprint(plan, lengths))
        return None if row is None else row["milliseconds"]


def native_plan(lengths: dict, limits: Constraints, cost: ProxyCost) -> Plan:
    rank_ids = replay(list(lengths.items()), limits.world, limits.token_cap, limits.min_cp, cost.beta_tokens)
    plan = from_rank_ids(rank_ids)
    validate(plan, lengths, limits)
    return plan


# ------------------------------------------------------------------ layout packing
class _Lpt:
    """One round of a fixed CP-size layout, filled longest sample first: each sample goes to the
    group that keeps the round's slowest group fastest (then the cheaper group, then the lower index)."""

    def __init__(self, sizes, lengths, limits, cost):
        self.lengths, self.limits, self.cost = lengths, limits, cost
        starts = [sum(sizes[:j]) for j in range(len(sizes))]
        self.groups = [Group(tuple(range(a, a + cp)), ()) for a, cp in zip(starts, sizes)]
        self.ms = [0.0] * len(sizes)

    def _allowed(self, ids, cp) -> bool:
        if not group_fits(ids, cp, self.lengths, self.limits):
            return False
        check = getattr(self.cost, "feasible_group", None)
        return check is None or check(ids, cp, self.lengths)

    def place(self, i) -> bool:
        best = None
        for j, g in enumerate(self.groups):
            ids = g.ids + (i,)
            if not self._allowed(ids, len(g.ranks)):
                continue
            new = self.cost.group(Group(g.ranks, ids), self.lengths)["cost"]
            others = max((v for k, v in enumerate(self.ms) if k != j), default=0)
            option = (max(new, others), self.ms[j], j, new)
            best = option if best is None or option < best else best
        if best is None:
            return False
        j, new = best[2], best[3]
        self.groups[j] = Group(self.groups[j].ranks, self.groups[j].ids + (i,))
        self.ms[j] = new
        return True


def pack_layout(lengths: dict, limits: Constraints, sizes: tuple[int, ...], cost) -> Plan:
    """LPT-pack the whole step into rounds of the CP-size vector ``sizes``. A round that would
    leave a group empty (ranks idle) is replaced by one world-wide group instead."""
    if sum(sizes) != limits.world:
        raise ValueError("Layout must cover the world")
    queue = sorted(lengths, key=lambda i: (-lengths[i], i))
    rounds = []
    while queue:
        lpt = _Lpt(sizes, lengths, limits, cost)
        rest = [i for i in queue if not lpt.place(i)]
        groups = lpt.groups
        if not all(g.ids for g in groups):
            taken, rest = [], []
            for i in queue:
                if group_fits(tuple(taken) + (i,), limits.world, lengths, limits):
                    taken.append(i)
                else:
                    rest.append(i)
            groups = [Group(tuple(range(limits.world)), tuple(taken))]
        if len(rest) == len(queue):
            raise ValueError("No feasible group for the next sequence")
        rounds.append(tuple(groups))
        queue = rest
    plan = tuple(rounds)
    validate(plan, lengths, limits)
    return plan


def layouts(limits: Constraints, seeds) -> list[tuple[int, ...]]:
    """CP-size vectors to pack: every homogeneous layout, every layout a seed plan uses, and
    each of those with one group halved or two equal aligned neighbours merged."""
    family = {(cp,) * (limits.world // cp) for cp in (1 << e for e in range(limits.world.bit_length()))
              if limits.min_cp <= cp <= limits.world}
    for plan in seeds:
        for batch in plan:
            sizes = tuple(len(g.ranks) for g in batch)
            family.add(sizes)
            for j, s in enumerate(sizes):
                if s > limits.min_cp:
                    family.add(sizes[:j] + (s // 2, s // 2) + sizes[j + 1:])
                mergeable = j + 1 < len(sizes) and sizes[j + 1] == s and sum(sizes[:j]) % (2 * s) == 0
                if mergeable:
                    family.add(sizes[:j] + (2 * s,) + sizes[j + 2:])
    return sorted(family)


# ------------------------------------------------------------------ local search
def neighbours(plan: Plan, lengths: dict, limits: Constraints):
    """Plans one step away from ``plan``, in a fixed order: first every move of one sample out of
    a group that keeps another sample into any other group of the step, then every swap of two
    samples of different lengths between two groups."""
    sites = [(m, j) for m, batch in enumerate(plan) for j in range(len(batch))]
    at = {site: plan[site[0]][site[1]] for site in sites}

    def edited(changes: dict) -> Plan:
        return tuple(tuple(changes.get((m, j), g) for j, g in enumerate(batch)) for m, batch in enumerate(plan))

    def fits(g: Group, ids) -> bool:
        return group_fits(ids, len(g.ranks), lengths, limits)

    for src in sites:
        a = at[src]
        if len(a.ids) < 2:
            continue
        for i in a.ids:
            kept = tuple(k for k in a.ids if k != i)
            for dst in sites:
                b = at[dst]
                if dst != src and fits(b, b.ids + (i,)):
                    yield edited({src: Group(a.ranks, kept), dst: Group(b.ranks, b.ids + (i,))})
    for x, src in enumerate(sites):
        a = at[src]
        for dst in sites[x + 1:]:
            b = at[dst]
            for i in a.ids:
                for k in b.ids:
                    if lengths[i] == lengths[k]:
                        continue
                    ids_a = tuple(k if n == i else n for n in a.ids)
                    ids_b = tuple(i if n == k else n for n in b.ids)
                    if fits(a, ids_a) and fits(b, ids_b):
                        yield edited({src: Group(a.ranks, ids_a), dst: Group(b.ranks, ids_b)})


def _improves(value: float, current: float) -> bool:
    """Strictly better beyond a relative 1e-9, so 1-ULP differences never decide."""
    return value < current - 1e-9 * max(1.0, abs(current))


class _Pool:
    """Legal candidate plans keyed by fingerprint; the first plan with a fingerprint keeps its name."""

    def __init__(self, lengths, limits, cost):
        self.lengths, self.limits, self.cost = lengths, limits, cost
        self.rows: dict[str, dict] = {}
        self.failures: list[dict] = []

    def add(self, name: str, plan: Plan) -> dict:
        validate(plan, self.lengths, self.limits)
        key = fingerprint(plan, self.lengths)
        if key not in self.rows:
            self.rows[key] = {"name": name, "plan": plan, "proxy_cost": self.cost.evaluate(plan, self.lengths),
                              "fingerprint": key}
        return self.rows[key]

    def attempt(self, name: str, make, label: str | None = None):
        try:
            return self.add(name, make())
        except (ValueError, AssertionError) as error:
            self.failures.append({"candidate": label or name, "reason": str(error)})
            return None

    def leader(self) -> dict:
        """Lowest proxy cost; insertion order (native first) breaks numerical ties."""
        rows = iter(self.rows.values())
        best = next(rows)
        for row in rows:
            if _improves(row["proxy_cost"], best["proxy_cost"]):
                best = row
        return best


def search(lengths: dict, limits: Constraints, cost, local_evaluations: int = 128, rounds: int = 2) -> dict:
    """A finite pool of legal plans and the best one under ``cost`` (see the module docstring)."""
    started = time.perf_counter()
    if local_evaluations < 0 or rounds < 0:
        raise ValueError("Search budgets must be nonnegative")
    pool = _Pool(lengths, limits, cost)
    seeds = []
    for name, proxy in (("native_square", ProxyCost("square", 1, 0)),
                        ("native_weighted", getattr(cost, "seed_proxy", cost))):
        row = pool.attempt(name, lambda proxy=proxy: native_plan(lengths, limits, proxy))
        if row is not None:
            seeds.append(row["plan"])
    for sizes in layouts(limits, seeds):
        name = "layout_" + "x".join(map(str, sizes))
        try:
            pool.add(name, pack_layout(lengths, limits, sizes, cost))
        except ValueError as error:
            pool.failures.append({"candidate": str(sizes), "reason": str(error)})
    if not pool.rows:
        raise ValueError("No legal candidate for this complete step")
    best, spent = pool.leader(), 0
    for _ in range(rounds):
        centre = best
        for plan in neighbours(centre["plan"], lengths, limits):
            if spent >= local_evaluations:
                break
            spent += 1
            try:
                row = pool.add("local_move_or_swap", plan)
            except ValueError as error:
                pool.failures.append({"candidate": "local_move_or_swap", "reason": str(error)})
                continue
            if _improves(cost.evaluate(plan, lengths), best["proxy_cost"]):
                best = row
        if best is centre or spent >= local_evaluations:
            break
    # a separate pass: moves cannot split the winner's rank domains into smaller CP groups
    from .short_sequence import refine_short_sequences
    refinement = refine_short_sequences(best["plan"], lengths, limits, cost)
    if refinement["plan"] != best["plan"]:
        best = pool.add("short_sequence_split", refinement["plan"])
    return {"selected": best, "candidates": list(pool.rows.values()), "failures": pool.failures,
            "local_evaluations": spent,
            "short_sequence_refinement": {k: v for k, v in refinement.items() if k != "plan"},
            "planning_ms": (time.perf_counter() - started) * 1000, "selection_provenance": cost.provenance,
            "parameter_sync_optimizer": "unknown"}


def select(result: dict, lengths: dict, measured: ExactCosts | None = None, allow_proxy: bool = False):
    """(candidate, basis): the fastest measured candidate when the table also measures the native
    plan, else the proxy's choice if explicitly allowed, else the native plan."""
    native = next((c for c in result["candidates"] if c["name"] == "native_square"), None)
    if measured and native is not None and measured.evaluate(native["plan"], lengths) is not None:
        timed = [(measured.evaluate(c["plan"], lengths), j) for j, c in enumerate(result["candidates"])]
        timed = [t for t in timed if t[0] is not None]
        return result["candidates"][min(timed)[1]], "measured_complete_plan"
    if allow_proxy:
        return result["selected"], "experimental_compute_proxy"
    if native is None:
        raise ValueError("Native plan is illegal; no calibrated fallback exists")
    return native, "native_fallback_unknown_distributed_cost"


def export_plan(plan: Plan, lengths: dict, cost: ProxyCost, node_size: int) -> dict:
    """Complete ownership, cost components and the per-rank Q / L imbalance of every microbatch."""
    batches = []
    for batch in plan:
        groups, per_rank_q, per_rank_l = [], [], []
        for g in batch:
            parts = cost.group(g, lengths)
            per_rank_q += [parts["q_ki2"]] * len(g.ranks)
            per_rank_l += [parts["l_ki"]] * len(g.ranks)
            nodes = {r // node_size for r in g.ranks}
            groups.append(dict(ranks=g.ranks, sample_ids=g.ids, padded_lengths=[lengths[i] for i in g.ids],
                               cp=len(g.ranks), placement="intra_node" if len(nodes) == 1 else "cross_node",
                               local_tokens=sum(lengths[i] for i in g.ids) / len(g.ranks), **parts))
        imbalance = lambda xs: max(xs) / (sum(xs) / len(xs))  # noqa: E731
        batches.append({"groups": groups, "cost": max(g["cost"] for g in groups), "r_q": imbalance(per_rank_q),
                        "r_l": imbalance(per_rank_l)})
    return {"microbatches": batches, "compute_proxy_cost": sum(b["cost"] for b in batches),
            "fingerprint": fingerprint(plan, lengths), "provenance": cost.provenance,
            "memory": "token_cap_only; measured_peak_required", "parameter_sync_optimizer": "unknown"}


def models(path: Path) -> dict[str, ProxyCost]:
    """Proxy models from a CP1 stack-coefficient table (gpt = 4 GQA, hybrid = 1 GQA + 3 GDN)."""
    rows = json.loads(Path(path).read_text())
    by_counts = {(r["gqa_layers"], r["gdn_layers"]): r for r in reversed(rows)}
    out = {"square": ProxyCost("square", 1.0, 0.0, "quadratic_work_proxy_Ki2")}
    for name, counts in (("gpt", (4, 0)), ("hybrid", (1, 3))):
        out[name] = ProxyCost(name, by_counts[counts]["A_ms_per_ki2"], by_counts[counts]["B_ms_per_ki"])
    return out
