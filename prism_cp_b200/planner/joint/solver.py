"""Joint microbatch packing x per-layer CP placement search.

The solver never consults the native N scheduler. It chooses (i) how the
samples of a global batch are packed into microbatches, (ii) for every
microbatch an ingress layout and, per layer, an attention layout (CP groups
and ranks; mode fixed by the kernel: GDN contiguous, GQA zigzag) and an MLP
placement, minimising the sum of predicted microbatch times plus the update,
under the whole forward/backward memory envelope of ``cost.Evaluator``.

* ``exact``   (<= 6 samples, <= 4 ranks): every aligned dyadic rank partition
  and sample assignment, a full DP over layer paths and a subset DP over the
  sample bitmask - optimal in the declared domain.
* ``bounded`` (default): candidate layouts from a bounded family (uniform CP,
  split-one-group, balanced heavy-CPp + CP1 tails, node-affine residency),
  a per-microbatch beam over layer paths that keeps both the fastest and the
  lowest-live-memory prefixes, and several complete pool packings proposed
  from memory-derived token targets; the best complete packing is the
  incumbent and is returned even when the state budget runs out.

The candidate families, beam rule and packing proposals are the reference's
(experiments/sequence_dynamic_cp/joint_cp/solver.py:20-458); they are kept
step-for-step so that the same inputs give the same plans and scores.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache
from itertools import product

from .cost import Evaluator, resource_metrics
from .ir import Group, Layout, Microbatch, Plan, validate_layout, validate_plan
from .memory_selection import prefer_lower_memory
from .response import ANCHOR_SCHEMAS, response_coverage


@dataclass(frozen=True)
class SearchOptions:
    mode: str = "bounded"
    beam: int = 8
    layouts: int = 8
    max_states: int = 1_000_000
    node_affinity: bool = False
    homogeneous_packing: bool = False
    balanced_packing: bool = False
    heavy_tail_packing: bool = False
    max_attention_cp: int | None = None
    memory_time_tolerance: float = 0.001

    def __post_init__(self):
        if self.mode not in ("exact", "bounded") or min(self.beam, self.layouts, self.max_states) < 1:
            raise ValueError("Invalid search options")
        c = self.max_attention_cp
        if c is not None and (c < 1 or c & (c - 1)):
            raise ValueError("Attention CP ceiling must be a positive power of two")
        if not math.isfinite(self.memory_time_tolerance) or self.memory_time_tolerance < 0:
            raise ValueError("Memory time tolerance must be finite and nonnegative")


class SearchLimit(RuntimeError):
    """Raised when the state budget is exhausted; no optimality claim survives it."""


@lru_cache(None)
def rank_partitions(start: int, width: int) -> tuple:
    """Every partition of ranks [start, start+width) into aligned dyadic intervals."""
    whole = ((tuple(range(start, start + width)),),)
    if width == 1:
        return whole
    half = width // 2
    return whole + tuple(a + b for a in rank_partitions(start, half) for b in rank_partitions(start + half, half))


def _make_layout(pairs) -> Layout:
    return Layout(tuple(Group(tuple(r), tuple(sorted(s))) for r, s in pairs), "zigzag")


def layout_candidates(ids, lengths, world, exact, limit, ranks_per_node=None, balanced_packing=False):
    ids = tuple(sorted(ids))
    found: list[Layout] = []
    seen: set = set()

    def add(pairs):
        lay = _make_layout(pairs)
        try:
            validate_layout(lay, lengths, world)
        except ValueError:
            return
        if lay not in seen:
            seen.add(lay)
            found.append(lay)

    if exact:
        for partition in rank_partitions(0, world):
            if len(partition) > len(ids):
                continue
            for assignment in product(range(len(partition)), repeat=len(ids)):
                packs = [[] for _ in partition]
                for s, j in zip(ids, assignment):
                    packs[j].append(s)
                add(zip(partition, packs))
        return found

    if ranks_per_node is not None and (ranks_per_node < 1 or ranks_per_node & (ranks_per_node - 1)):
        raise ValueError("Node-affine candidate groups require a power-of-two node size")

    def assign(order, partition):
        packs, loads = [[] for _ in partition], [0.0] * len(partition)
        for s in order:
            legal = [j for j, r in enumerate(partition) if len(r) == 1 or lengths[s] % (2 * len(r)) == 0]
            if not legal:
                return None
            j = min(legal, key=lambda j: (bool(packs[j]), loads[j], j))
            packs[j].append(s)
            loads[j] += lengths[s] / len(partition[j])
        return packs

    heavy_first = sorted(ids, key=lambda s: (-lengths[s], s))
    if balanced_packing:
        # one CPp group for the heavy samples plus CP1 tails, anchored at either end
        width = world // 2
        while width > 1:
            for start in (0, world - width):
                big = tuple(range(start, start + width))
                partition = (big,) + tuple((r,) for r in range(world) if r not in big)
                if len(partition) <= len(ids):
                    packs = assign(heavy_first, partition)
                    if packs is not None:
                        add(sorted(zip(partition, packs)))
            width //= 2

    partitions = []
    width = world
    while width:
        uniform = tuple(tuple(range(i, i + width)) for i in range(0, world, width))
        partitions.append(uniform)
        if width > 1 and len(uniform) < len(ids):
            for pick in (0, len(uniform) - 1):
                r = uniform[pick]
                h = width // 2
                partitions.append(uniform[:pick] + (r[:h], r[h:]) + uniform[pick + 1:])
        width //= 2
    for partition in partitions:
        if len(partition) > len(ids):
            continue
        for order in (heavy_first, list(ids), list(reversed(ids))):
            node_local = (ranks_per_node is not None and world > ranks_per_node
                          and all(r[0] // ranks_per_node == r[-1] // ranks_per_node for r in partition))
            if node_local:
                # keep each sample's node fixed across CP widths (no inter-node reshard)
                nodes = tuple(tuple(range(s, min(s + ranks_per_node, world))) for s in range(0, world, ranks_per_node))
                buckets = assign(order, nodes)
                packs = None
                if buckets is not None:
                    packs = []
                    for node, samples in zip(nodes, buckets):
                        sub = tuple(r for r in partition if r[0] in node)
                        placed = assign(samples, sub)
                        if placed is None:
                            packs = None
                            break
                        packs.extend(placed)
            else:
                packs = assign(order, partition)
            if packs is not None:
                add(zip(partition, packs))
    if len(found) <= limit:
        return found
    uniform = [x for x in found if len({len(g.ranks) for g in x.groups}) == 1]
    varied = [x for x in found if x not in uniform]
    picked, widths = [], set()
    for lay in uniform:
        w = len(lay.groups[0].ranks)
        if w not in widths:
            picked.append(lay)
            widths.add(w)
    rest = varied + [x for x in uniform if x not in picked]
    return (picked + rest)[:limit]


@dataclass(frozen=True)
class _State:
    cost: float
    live: tuple
    peak: tuple
    ingress: Layout
    previous: Layout
    layers: tuple


class _Search:
    def __init__(self, lengths, world, pattern, model, options):
        self.lengths, self.world, self.pattern = lengths, world, pattern
        self.model, self.options = model, options
        self.states = 0
        self.truncated = False
        self.cache: dict = {}
        self.incumbent = None
        self.packings_examined = 0

    def batch(self, ids):
        """Best microbatch for these samples; solved once per length shape."""
        ids = tuple(sorted(ids))
        shape = tuple(self.lengths[i] for i in ids)
        if shape not in self.cache:
            self.cache[shape] = self._batch(dict(enumerate(shape)))
        answer = self.cache[shape]
        if answer is None:
            return None
        cost, mb = answer

        def remap(lay):
            return Layout(tuple(Group(g.ranks, tuple(ids[s] for s in g.samples)) for g in lay.groups), lay.mode)

        return cost, Microbatch(remap(mb.ingress), tuple((remap(a), remap(m)) for a, m in mb.layers))

    def _batch(self, lengths):
        opt, m = self.options, self.model
        if sum(lengths.values()) > m.token_capacity_upper_bound(self.pattern, self.world):
            return None
        cands = layout_candidates(lengths, lengths, self.world, opt.mode == "exact", opt.layouts,
                                  m.ranks_per_node if opt.node_affinity else None, opt.balanced_packing)
        ev = Evaluator(m, lengths, self.world, self.pattern)
        mlps = tuple(dict.fromkeys(x.with_mode(md) for x in cands for md in ("contiguous", "zigzag")))
        attn = [x for x in cands if opt.max_attention_cp is None
                or all(len(g.ranks) <= opt.max_attention_cp for g in x.groups)]
        if m.cp_response and m.cp_response.get("schema") in ANCHOR_SCHEMAS:
            ceiling = max(int(c) for c in m.cp_response["anchors"]["GQA"]["milliseconds"])
            if m.cp_response["schema"] != "h100_operator_anchors_v1":
                attn = [x for x in attn if all(str(len(g.ranks)) in m.cp_response["anchors"]["GQA"]["milliseconds"]
                                               for g in x.groups)]
            attn = [x for x in attn if all(len(g.ranks) <= ceiling for g in x.groups)]
        states = [_State(0.0, ev.initial(x), ev.initial(x), x, x, ()) for x in cands
                  if max(ev.initial(x)) <= m.budget]
        for symbol in self.pattern:
            nxt = []
            for st in states:
                for template in attn:
                    a = template.with_mode("contiguous" if symbol == "G" else "zigzag")
                    for mlp in mlps:
                        self.states += 1
                        if self.states > opt.max_states:
                            raise SearchLimit("Search state budget exhausted; no global optimum is certified")
                        cost, live, here = ev.layer(st.live, st.previous, a, mlp, symbol)
                        peak = tuple(max(x, y) for x, y in zip(st.peak, here))
                        if max(peak) <= m.budget:
                            nxt.append(_State(st.cost + cost, live, peak, st.ingress, a, st.layers + ((a, mlp),)))
            if opt.mode == "bounded" and len(nxt) > opt.beam:
                self.truncated = True
                fastest = sorted(nxt, key=lambda s: (s.cost, max(s.peak)))
                safest = sorted(nxt, key=lambda s: (max(s.live), s.cost))
                keep: dict = {}
                for pair in zip(fastest, safest):
                    for s in pair:
                        sig = (s.ingress, s.previous, s.live)
                        if sig not in keep or s.cost < keep[sig].cost:
                            keep[sig] = s
                        if len(keep) >= opt.beam:
                            break
                    if len(keep) >= opt.beam:
                        break
                nxt = list(keep.values())
            states = nxt
        best = None
        for st in states:
            cost, head = ev.finish(st.live, st.previous, st.ingress)
            if max(head) <= m.budget:
                row = (st.cost + cost, Microbatch(st.ingress, st.layers))
                if best is None or row[0] < best[0]:
                    best = row
        return best

    def exact(self):
        ids = tuple(sorted(self.lengths))

        @lru_cache(None)
        def visit(mask):
            if not mask:
                return 0.0, ()
            low = mask & -mask
            best = None
            sub = mask
            while sub:
                if sub & low:
                    chosen = tuple(ids[i] for i in range(len(ids)) if sub & (1 << i))
                    row = self.batch(chosen)
                    if row is not None:
                        rest = visit(mask ^ sub)
                        if rest is not None:
                            cand = (row[0] + rest[0], (row[1],) + rest[1])
                            if best is None or cand[0] < best[0]:
                                best = cand
                sub = (sub - 1) & mask
            return best

        return visit((1 << len(ids)) - 1)

    def _greedy_packs(self, order, target, first=()):
        packs = [tuple(sorted(first))] if first else []
        pack, total = [], 0
        for s in order:
            if pack and total + self.lengths[s] > target:
                packs.append(tuple(sorted(pack)))
                pack, total = [], 0
            pack.append(s)
            total += self.lengths[s]
        if pack:
            packs.append(tuple(sorted(pack)))
        return tuple(packs)

    def bounded(self):
        m, L = self.model, self.lengths
        ev = Evaluator(m, L, self.world, self.pattern)
        h, f, d = m.hidden, m.ffn, m.gdn_heads * m.gdn_dim
        per_token = 4 * h + len(self.pattern) * 2 * (12 * h + 3 * f + max(5 * d, h + 2 * m.kv_heads * m.head_dim))
        nominal = max(1, int((m.budget - ev.base) / per_token)) * self.world
        longest = max(L.values())
        targets = {max(longest, int(nominal * k)) for k in (0.5, 0.8, 1.0, 1.3)}
        quantum = self.world * math.gcd(*L.values())
        targets.update(max(longest, (t // quantum) * quantum) for t in tuple(targets))
        targets = sorted(targets)
        orders = [tuple(sorted(L)), tuple(sorted(L, key=lambda s: (-L[s], s)))]
        proposals = [self._greedy_packs(o, t) for o in orders for t in targets]
        if self.options.homogeneous_packing:
            buckets: dict = {}
            for s in sorted(L):
                buckets.setdefault(L[s], []).append(s)
            for t in targets:
                packs = []
                for n, samples in sorted(buckets.items(), reverse=True):
                    c = max(1, t // n)
                    packs.extend(tuple(samples[i:i + c]) for i in range(0, len(samples), c))
                proposals.append(tuple(packs))
        if self.options.balanced_packing:
            order = sorted(L, key=lambda s: (-L[s], s))
            anchor, tail = order[0], sorted(order[1:], key=lambda s: (L[s], s))
            balanced = []
            width = self.world // 2
            while width:
                if width == 1 or L[anchor] % (2 * width) == 0:
                    goal = L[anchor] * (self.world - width) / width
                    picked, tok = [], 0
                    for s in tail:
                        if tok + L[s] <= goal:
                            picked.append(s)
                            tok += L[s]
                    if len(picked) >= self.world - width:
                        paired = frozenset((anchor, *picked))
                        rest = tuple(s for s in order if s not in paired)
                        balanced.extend(self._greedy_packs(rest, t, first=paired) for t in targets)
                width //= 2
            proposals = balanced + proposals
        if self.options.heavy_tail_packing:
            ceiling = m.token_capacity_upper_bound(self.pattern, self.world)
            smallest = min(L.values())
            heavy = sorted((s for s in L if L[s] >= longest / 2), key=lambda s: (-L[s], s))
            hs = set(heavy)
            tail = sorted((s for s in L if s not in hs), key=lambda s: (L[s], s))
            extra_props = []
            if tail and longest >= 4 * smallest:
                top = min(len(heavy), self.world // m.ranks_per_node, ceiling // longest)
                for count in range(1, top + 1):
                    blocks = [heavy[i:i + count] for i in range(0, len(heavy), count)]
                    for extra in sorted({0, 1, 2, 4, 8, 16, 32, len(tail) // len(blocks)}):
                        for t in targets:
                            packs, cursor = [], 0
                            for block in blocks:
                                pack, total = list(block), sum(L[s] for s in block)
                                for _ in range(extra):
                                    if cursor == len(tail) or total + L[tail[cursor]] > ceiling:
                                        break
                                    pack.append(tail[cursor])
                                    total += L[tail[cursor]]
                                    cursor += 1
                                packs.append(tuple(sorted(pack)))
                            packs.extend(self._greedy_packs(tail[cursor:], t))
                            extra_props.append(tuple(packs))
            proposals = extra_props + proposals
        seen, best = set(), None
        for sig in proposals:
            if sig in seen:
                continue
            seen.add(sig)
            self.packings_examined += 1
            rows = []
            for ids in sig:
                row = self.batch(ids)
                if row is None:
                    break
                rows.append(row)
            else:
                ans = (sum(r[0] for r in rows), tuple(r[1] for r in rows))
                if best is None or ans[0] < best[0]:
                    best = ans
                    self.incumbent = best
        return best


def solve(lengths: dict, world: int, pattern: str, model, options: SearchOptions = SearchOptions()) -> dict:
    if (not lengths or world <= 0 or world & (world - 1) or not pattern or set(pattern) - set("G*")
            or any(type(s) is not int or type(n) is not int or n <= 0 for s, n in lengths.items())):
        raise ValueError("Invalid lengths, world or pattern")
    if options.mode == "exact" and (len(lengths) > 6 or world > 4):
        raise ValueError("Exact domain is limited to <=6 samples and <=4 ranks; use bounded mode")
    search = _Search(lengths, world, pattern, model, options)
    limit_hit = False
    try:
        answer = search.exact() if options.mode == "exact" else search.bounded()
    except SearchLimit:
        if options.mode == "exact":
            raise
        limit_hit = True
        answer = search.incumbent
    meta = {"search_mode": options.mode, "states_examined": search.states, "state_budget_exhausted": limit_hit,
            "pool_packings_examined": search.packings_examined, "microbatch_shapes_solved": len(search.cache),
            "beam_pruned": search.truncated,
            "domain": "aligned dyadic groups; ascending sample order per pack; all ranks nonempty; no padding; "
                      "fixed G/* kernel modes; independent MLP placement",
            "objective": "minimize allocated GPU-ms for fixed useful input work; fixed world makes this equivalent "
                         "to sum complete F+B microbatch times plus update/sync; all allocated ranks and idle waits "
                         "counted",
            "model_provenance": model.provenance, "gpu_admitted": False,
            "max_attention_cp": options.max_attention_cp}
    if answer is None:
        status = ("search_budget_exhausted" if limit_hit else
                  "infeasible_in_declared_domain" if options.mode == "exact" else "no_feasible_plan_found")
        return dict(meta, status=status, plan=None)
    plan = Plan(world, pattern, answer[1])
    validate_plan(plan, lengths)
    ev = Evaluator(model, lengths, world, pattern)
    evidence = [ev.evaluate(b) for b in plan.microbatches]
    if not all(r["fits"] for r in evidence):
        raise AssertionError("Solver and full-plan memory accounting disagree")
    total = sum(r["predicted_ms"] for r in evidence) + model.update_ms
    if not math.isclose(total, answer[0] + model.update_ms, rel_tol=1e-10, abs_tol=1e-8):
        raise AssertionError("Solver and full-plan objective disagree")
    if options.mode == "bounded":
        plan, meta["memory_selection"] = prefer_lower_memory(plan, lengths, model, options.memory_time_tolerance)
        validate_plan(plan, lengths)
        ev = Evaluator(model, lengths, world, pattern)
        evidence = [ev.evaluate(b) for b in plan.microbatches]
        total = sum(r["predicted_ms"] for r in evidence) + model.update_ms
        meta["objective"] += "; bounded CP1 memory tie-break within declared time tolerance"
    return dict(meta, status="optimal_in_declared_domain" if options.mode == "exact"
                else "best_found_no_optimality_certificate",
                plan=plan.to_dict(), predicted_update_ms=total,
                resource_metrics=resource_metrics(lengths, world, pattern, model, total),
                cp_response_evidence=response_coverage(plan, lengths, model),
                budget_bytes=model.budget, microbatch_evidence=evidence)
