"""Online per-batch CP selection (new capability; the reference left it unimplemented).

For every global batch, before it runs, choose a CP degree separately for the
GDN and the GQA layers from ``degrees`` (default {1, 2, 4, 8}) and pack the
documents into microbatches, scoring each candidate plan with the joint cost
and memory model (``joint.cost.Evaluator``, optionally calibrated by a B200
response profile). Candidates:

* ``(cp_gdn, cp_gqa)`` for every pair of degrees: documents are packed longest
  first into microbatches whose per-rank tokens stay within the memory-derived
  capacity at the larger degree; GDN layers use ``world / cp_gdn`` contiguous
  teams, GQA layers ``world / cp_gqa`` zigzag teams over the same samples, so
  every GDN<->GQA boundary with different degrees is a CP-transition reshard;
* documents longer than a team can hold at a degree raise that degree for the
  batch (the degree is the minimum that fits the longest document); with
  ``Model.recompute_tokens`` set, such a document may instead run alone in a
  microbatch that recomputes every layer in the backward, priced as such.

* dynamic plans: the CP degree chosen per document by the dynamic-CP
  scheduler at a few per-rank capacities (teams of different sizes side by
  side in one microbatch, short documents on CP1 ranks), kept when the model
  predicts them faster than every uniform pair.

The selection is deterministic (same lengths -> same plan on every rank), costs
milliseconds of CPU per batch, and returns the plan with its predicted update
time and the degree pair, so the executor can apply it without touching
process groups (all dyadic teams exist from start-up).
"""

from __future__ import annotations

from dataclasses import dataclass

from .joint.cost import Evaluator, Model
from .joint.ir import Group, Layout, Microbatch, Plan, validate_plan


@dataclass(frozen=True)
class Selection:
    plan: Plan
    cp_gdn: int          # 0 for a dynamic plan (CP chosen per document)
    cp_gqa: int
    predicted_update_ms: float
    candidates: tuple
    dynamic_capacity: int | None = None   # per-rank token capacity of a dynamic plan

    @property
    def description(self) -> str:
        if self.dynamic_capacity is not None:
            return f"dynamic CP per document (K = {self.dynamic_capacity})"
        return f"cp_gdn{self.cp_gdn} cp_gqa{self.cp_gqa}"


def _pack(lengths: dict, order, capacity_tokens: int, groups: int):
    """Greedy longest-first packing into microbatches of ``groups`` bins of
    ``capacity_tokens`` tokens each (a bin = one team's share of the world)."""
    batches = []
    pending = list(order)
    while pending:
        bins = [[] for _ in range(groups)]
        loads = [0] * groups
        rest = []
        for s in pending:
            j = min(range(groups), key=lambda i: (loads[i], i))
            if loads[j] + lengths[s] <= capacity_tokens or not bins[j]:
                bins[j].append(s)
                loads[j] += lengths[s]
            else:
                rest.append(s)
        if any(not b for b in bins):
            merged = sorted(s for b in bins for s in b)
            bins = [merged]
        batches.append([tuple(sorted(b)) for b in bins])
        if len(rest) == len(pending):
            raise ValueError("no progress while packing")
        pending = rest
    return batches


def _split(samples, lengths, parts: int):
    bins = [[] for _ in range(parts)]
    loads = [0] * parts
    for s in sorted(samples, key=lambda s: (-lengths[s], s)):
        j = min(range(parts), key=lambda i: (loads[i], i))
        bins[j].append(s)
        loads[j] += lengths[s]
    if any(not b for b in bins):
        return None
    return [tuple(sorted(b)) for b in bins]


def candidate_plan(lengths: dict, world: int, pattern: str, cp_gdn: int, cp_gqa: int, capacity: int,
                   oversize: bool = False):
    """Plan with GDN teams of ``cp_gdn`` and GQA teams of ``cp_gqa`` ranks, or None. With
    ``oversize`` a document longer than a team's capacity still gets a microbatch of its own
    (the evaluator then prices it with per-layer recompute, if the model allows that)."""
    coarse = max(cp_gdn, cp_gqa)
    fine = min(cp_gdn, cp_gqa)
    for n in lengths.values():
        if coarse > 1 and n % (2 * coarse):
            return None
        if fine > 1 and n % (2 * fine):
            return None
    order = sorted(lengths, key=lambda s: (-lengths[s], s))
    if max(lengths.values()) > capacity * coarse and not oversize:
        return None
    mbs = []
    for coarse_bins in _pack(lengths, order, capacity * coarse, world // coarse):
        if len(coarse_bins) != world // coarse:
            return None
        fine_bins = []
        ratio = coarse // fine
        for b in coarse_bins:
            parts = _split(b, lengths, ratio) if ratio > 1 else [b]
            if parts is None:
                return None
            if not oversize and any(sum(lengths[s] for s in p) > capacity * fine for p in parts):
                return None
            fine_bins.extend(parts)
        def lay(cp, bins, mode):
            return Layout(tuple(Group(tuple(range(i * cp, (i + 1) * cp)), tuple(b)) for i, b in enumerate(bins)),
                          mode)
        g_bins = coarse_bins if cp_gdn == coarse else fine_bins
        a_bins = coarse_bins if cp_gqa == coarse else fine_bins
        gdn = lay(cp_gdn, g_bins, "contiguous")
        gqa = lay(cp_gqa, a_bins, "zigzag")
        layers = tuple((gdn, gdn) if c == "G" else (gqa, gqa) for c in pattern)
        mbs.append(Microbatch(gqa, layers))
    plan = Plan(world, pattern, tuple(mbs))
    validate_plan(plan, lengths)
    return plan


def _packing_threshold(model: Model) -> int | None:
    """Per-rank tokens above which a microbatch recomputes, when that is a threshold (packing keeps
    ordinary microbatches below it); None when nothing recomputes or everything does (0: full
    recompute, where the memory model alone bounds the capacity)."""
    r = model.recompute_tokens
    return r if r is not None and r > 0 else None


def dynamic_candidates(lengths: dict, world: int, pattern: str, model: Model,
                       capacities=(16384, 24576, 32768)) -> list[tuple]:
    """Plans with the CP degree chosen per document (the dynamic-CP scheduler at per-rank token
    capacity K: a document gets the smallest dyadic team that holds it, short documents share CP1
    ranks, teams of different sizes run side by side in one microbatch), as
    ``(predicted ms, K, plan, rows)`` of the candidates that fit."""
    from .studies import native_joint_plan
    ev = Evaluator(model, lengths, world, pattern)
    out = []
    threshold = _packing_threshold(model)
    for cap in capacities:
        if threshold is not None and cap > threshold:
            continue
        try:
            plan = native_joint_plan(lengths, world, pattern, cap)
        except ValueError:
            continue
        evid = [ev.evaluate(mb) for mb in plan.microbatches]
        if all(e["fits"] for e in evid):
            ms = sum(e["predicted_ms"] for e in evid) + model.update_ms
            out.append((ms, cap, plan, {"dynamic_capacity": cap, "fits": True, "predicted_update_ms": ms,
                                        "microbatches": len(plan.microbatches)}))
    return out


def select(lengths: dict, world: int, pattern: str, model: Model, degrees=(1, 2, 4, 8),
           capacity: int | None = None, dynamic: bool = True) -> Selection:
    """Best plan for this batch under ``model``: a (cp_gdn, cp_gqa) pair for all documents, or
    (with ``dynamic``) a per-document CP plan when the model predicts it faster."""
    degrees = tuple(d for d in degrees if d <= world and world % d == 0)
    if dynamic and world > 1:
        try:
            uniform = select(lengths, world, pattern, model, degrees, capacity, dynamic=False)
        except ValueError:
            uniform = None
        best = min(dynamic_candidates(lengths, world, pattern, model), default=None, key=lambda c: (c[0], c[1]))
        if best is not None and (uniform is None or best[0] < uniform.predicted_update_ms):
            rows = (uniform.candidates if uniform is not None else ()) + (best[3],)
            return Selection(best[2], 0, 0, best[0], rows, best[1])
        if uniform is None:
            raise ValueError("no candidate plan fits this batch")
        return uniform
    if capacity is None:
        # the memory model's token ceiling is necessary, not sufficient (CP workspaces come on top):
        # shrink the per-rank capacity until some candidate fits
        top = max(1, model.token_capacity_upper_bound(pattern, world) // world)
        threshold = _packing_threshold(model)
        if threshold is not None:
            # pack ordinary microbatches below the recompute threshold; only documents longer than
            # a team's share run alone with recompute
            top = min(top, threshold)
        last = None
        for frac in (1.0, 0.9, 0.8, 0.7, 0.6, 0.5, 0.4, 0.3):
            try:
                return select(lengths, world, pattern, model, degrees, max(1, int(top * frac)), dynamic=False)
            except ValueError as err:
                last = err
        raise last
    ev = Evaluator(model, lengths, world, pattern)
    rows = []
    best = None
    for cg in degrees:
        for ca in degrees:
            try:
                plan = candidate_plan(lengths, world, pattern, cg, ca, capacity,
                                      oversize=model.recompute_tokens is not None)
            except ValueError:
                plan = None
            if plan is None:
                continue
            evid = [ev.evaluate(mb) for mb in plan.microbatches]
            if not all(e["fits"] for e in evid):
                rows.append({"cp_gdn": cg, "cp_gqa": ca, "fits": False})
                continue
            ms = sum(e["predicted_ms"] for e in evid) + model.update_ms
            rows.append({"cp_gdn": cg, "cp_gqa": ca, "fits": True, "predicted_update_ms": ms,
                         "microbatches": len(plan.microbatches),
                         "recomputed_microbatches": sum(bool(e.get("recompute")) for e in evid)})
            key = (ms, cg, ca)
            if best is None or key < best[0]:
                best = (key, plan, cg, ca, ms)
    if best is None:
        raise ValueError("no candidate CP pair fits this batch")
    _, plan, cg, ca, ms = best
    return Selection(plan, cg, ca, ms, tuple(rows))
