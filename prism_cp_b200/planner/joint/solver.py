"""Joint microbatch packing x per-layer CP placement search.

The solver never consults the native N scheduler. For a global batch it chooses
(i) how the samples are packed into microbatches and (ii) for every microbatch
an ingress layout and, per layer, an attention layout (CP groups and their
ranks; the kernel fixes the mode: GDN contiguous, GQA zigzag) and an MLP
placement. The objective is the sum of predicted microbatch times plus the
update, subject to the per-rank forward/backward memory envelope of
``cost.Evaluator``.

* ``exact`` (<= 6 samples, <= 4 ranks): every aligned dyadic rank partition and
  sample assignment, every layer path, and a DP over sample subsets - optimal
  in the declared domain.
* ``bounded`` (default): layouts from a bounded family (uniform CP, one group
  split, a heavy CPp group with CP1 tails, node-affine residency), a beam over
  layer paths that keeps the fastest and the lowest-live-memory prefixes, and
  a list of complete pool packings proposed from memory-derived token
  targets. The best complete packing seen is the incumbent and survives an
  exhausted state budget.

The candidate families, the beam's keep rule, the packing proposals and every
tie-break are the reference's (joint_cp/solver.py:20-458) so that the same
inputs give the same plans and scores; the code is organised differently: a
``_Layouts`` builder per microbatch shape, a ``_PathSearch`` over layer paths,
and proposal generators that each yield candidate packings.
"""

from __future__ import annotations

import itertools
import math
from dataclasses import dataclass
from functools import lru_cache

from .cost import Evaluator, resource_metrics
from .ir import Group, Layout, Microbatch, Plan, validate_layout, validate_plan
from .memory_selection import prefer_lower_memory
from .response import profile_of, response_coverage


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
        ceiling = self.max_attention_cp
        if ceiling is not None and not (ceiling >= 1 and ceiling & (ceiling - 1) == 0):
            raise ValueError("Attention CP ceiling must be a positive power of two")
        if not (math.isfinite(self.memory_time_tolerance) and self.memory_time_tolerance >= 0):
            raise ValueError("Memory time tolerance must be finite and nonnegative")


class SearchLimit(RuntimeError):
    """Raised when the state budget is exhausted; no optimality claim survives it."""


@lru_cache(None)
def rank_partitions(start: int, width: int) -> tuple:
    """Every partition of ranks [start, start + width) into aligned dyadic intervals: the whole
    interval first, then every partition of the left half combined with every one of the right."""
    whole = (tuple(range(start, start + width)),)
    if width == 1:
        return (whole,)
    half = width // 2
    pairs = itertools.product(rank_partitions(start, half), rank_partitions(start + half, half))
    return (whole,) + tuple(left + right for left, right in pairs)


# ------------------------------------------------------------------ candidate layouts
class _Layouts:
    """Ordered, deduplicated, validated zigzag layouts of one microbatch's samples."""

    def __init__(self, lengths: dict, world: int):
        self.lengths, self.world = lengths, world
        self.items: list[Layout] = []
        self._seen: set = set()

    def add(self, partition, packs) -> None:
        layout = Layout(tuple(Group(tuple(r), tuple(sorted(p))) for r, p in zip(partition, packs)), "zigzag")
        try:
            validate_layout(layout, self.lengths, self.world)
        except ValueError:
            return
        if layout not in self._seen:
            self._seen.add(layout)
            self.items.append(layout)

    def fill(self, order, partition):
        """Greedy fill: each sample (in ``order``) goes to a legal group (CP1, or one whose
        zigzag divides it) - an empty one first, then the least loaded per rank, then the
        lowest index. None if some sample has no legal group."""
        packs = [[] for _ in partition]
        load = [0.0] * len(partition)
        for s in order:
            legal = [j for j, ranks in enumerate(partition)
                     if len(ranks) == 1 or self.lengths[s] % (2 * len(ranks)) == 0]
            if not legal:
                return None
            j = min(legal, key=lambda j: (len(packs[j]) > 0, load[j], j))
            packs[j].append(s)
            load[j] += self.lengths[s] / len(partition[j])
        return packs

    def fill_by_node(self, order, partition, nodes):
        """``fill`` onto whole nodes first, then onto the partition's groups inside each node
        (samples keep their node for every CP width of the family)."""
        per_node = self.fill(order, nodes)
        if per_node is None:
            return None
        packs = []
        for node, samples in zip(nodes, per_node):
            placed = self.fill(samples, tuple(r for r in partition if r[0] in node))
            if placed is None:
                return None
            packs += placed
        return packs


def _cheap_partitions(world: int, samples: int):
    """Uniform partitions of every dyadic width, each followed (when there are more samples than
    groups) by the variants with its first or its last group split in two."""
    width = world
    while width:
        uniform = tuple(tuple(range(i, i + width)) for i in range(0, world, width))
        yield uniform
        if width > 1 and len(uniform) < samples:
            half = width // 2
            for j in (0, len(uniform) - 1):
                yield uniform[:j] + (uniform[j][:half], uniform[j][half:]) + uniform[j + 1:]
        width //= 2


def _heavy_plus_singles(world: int):
    """One CP-p group (p = world/2 .. 2) at either end of the world, every other rank CP1."""
    width = world // 2
    while width > 1:
        for start in (0, world - width):
            big = tuple(range(start, start + width))
            yield (big,) + tuple((r,) for r in range(world) if r not in big)
        width //= 2


def _shortlist(found: list[Layout], limit: int) -> list[Layout]:
    """At most ``limit`` layouts: one uniform layout per CP width first (no attention costs are
    consulted), then the heterogeneous placements, then the remaining uniform ones."""
    if len(found) <= limit:
        return found
    uniform = [x for x in found if len({len(g.ranks) for g in x.groups}) == 1]
    first_per_width = {}
    for x in uniform:
        first_per_width.setdefault(len(x.groups[0].ranks), x)
    head = list(first_per_width.values())
    tail = [x for x in found if x not in uniform] + [x for x in uniform if x not in head]
    return (head + tail)[:limit]


def layout_candidates(ids, lengths, world, exact, limit, ranks_per_node=None, balanced_packing=False):
    ids = tuple(sorted(ids))
    out = _Layouts(lengths, world)
    if exact:
        for partition in rank_partitions(0, world):
            if len(partition) > len(ids):
                continue
            for owner in itertools.product(range(len(partition)), repeat=len(ids)):
                out.add(partition, [[s for s, j in zip(ids, owner) if j == k] for k in range(len(partition))])
        return out.items
    if ranks_per_node is not None and not (ranks_per_node >= 1 and ranks_per_node & (ranks_per_node - 1) == 0):
        raise ValueError("Node-affine candidate groups require a power-of-two node size")
    heavy_first = sorted(ids, key=lambda s: (-lengths[s], s))
    if balanced_packing:
        for partition in _heavy_plus_singles(world):
            if len(partition) <= len(ids):
                packs = out.fill(heavy_first, partition)
                if packs is not None:
                    pairs = sorted(zip(partition, packs))
                    out.add([r for r, _ in pairs], [p for _, p in pairs])
    nodes = None
    if ranks_per_node is not None and world > ranks_per_node:
        nodes = tuple(tuple(range(a, min(a + ranks_per_node, world))) for a in range(0, world, ranks_per_node))
    for partition in _cheap_partitions(world, len(ids)):
        if len(partition) > len(ids):
            continue
        node_local = nodes is not None and all(r[0] // ranks_per_node == r[-1] // ranks_per_node
                                               for r in partition)
        for order in (heavy_first, list(ids), list(reversed(ids))):
            packs = out.fill_by_node(order, partition, nodes) if node_local else out.fill(order, partition)
            if packs is not None:
                out.add(partition, packs)
    return _shortlist(out.items, limit)


# ------------------------------------------------------------------ layer paths of one microbatch
@dataclass(frozen=True)
class _Path:
    """A prefix of layer choices of one microbatch and its memory state."""

    cost: float
    live: tuple
    peak: tuple
    ingress: Layout
    previous: Layout
    layers: tuple


def _beam(paths: list[_Path], width: int) -> list[_Path]:
    """Keep ``width`` prefixes, alternating between the fastest (cost, peak) and the lowest live
    memory (live, cost) ranking; prefixes that end in the same state keep the cheaper one."""
    by_time = sorted(paths, key=lambda p: (p.cost, max(p.peak)))
    by_memory = sorted(paths, key=lambda p: (max(p.live), p.cost))
    kept: dict = {}
    for p in itertools.chain.from_iterable(zip(by_time, by_memory)):
        state = (p.ingress, p.previous, p.live)
        held = kept.get(state)
        if held is None or p.cost < held.cost:
            kept[state] = p
        if len(kept) >= width:
            break
    return list(kept.values())


class _PathSearch:
    """Best (cost, microbatch) of one microbatch's samples over its candidate layouts."""

    def __init__(self, owner: "_Search", lengths: dict):
        self.owner, self.lengths = owner, lengths
        o, m = owner.options, owner.model
        self.budget = m.budget
        self.ev = Evaluator(m, lengths, owner.world, owner.pattern)
        self.layouts = layout_candidates(lengths, lengths, owner.world, o.mode == "exact", o.layouts,
                                         m.ranks_per_node if o.node_affinity else None, o.balanced_packing)
        # the MLP can stay in the attention ownership or take any candidate placement, in either mode
        self.mlps = tuple(dict.fromkeys(x.with_mode(mode) for x in self.layouts for mode in ("contiguous", "zigzag")))
        profile = profile_of(m)

        def attention_ok(layout):
            degrees = {len(g.ranks) for g in layout.groups}
            if o.max_attention_cp is not None and max(degrees) > o.max_attention_cp:
                return False
            return all(profile.allows_attention_cp(d) for d in degrees)

        self.attention = [x for x in self.layouts if attention_ok(x)]

    def _extend(self, paths: list[_Path], symbol: str) -> list[_Path]:
        mode = "contiguous" if symbol == "G" else "zigzag"
        out = []
        for p in paths:
            for template in self.attention:
                attention = template.with_mode(mode)
                for mlp in self.mlps:
                    self.owner.count_state()
                    ms, live, here = self.ev.layer(p.live, p.previous, attention, mlp, symbol)
                    peak = tuple(map(max, p.peak, here))
                    if max(peak) <= self.budget:
                        out.append(_Path(p.cost + ms, live, peak, p.ingress, attention, p.layers + ((attention, mlp),)))
        return out

    def run(self):
        start = [(x, self.ev.initial(x)) for x in self.layouts]
        paths = [_Path(0, live, live, x, x, ()) for x, live in start if max(live) <= self.budget]
        width = self.owner.options.beam
        for symbol in self.owner.pattern:
            paths = self._extend(paths, symbol)
            if self.owner.options.mode == "bounded" and len(paths) > width:
                self.owner.truncated = True
                paths = _beam(paths, width)
        best = None
        for p in paths:
            ms, head = self.ev.finish(p.live, p.previous, p.ingress)
            if max(head) <= self.budget and (best is None or p.cost + ms < best[0]):
                best = (p.cost + ms, Microbatch(p.ingress, p.layers))
        return best


def _relabel(mb: Microbatch, ids: tuple) -> Microbatch:
    """A microbatch solved on local sample indices 0..n-1, with the real sample ids."""
    def lay(x: Layout) -> Layout:
        return Layout(tuple(Group(g.ranks, tuple(ids[s] for s in g.samples)) for g in x.groups), x.mode)
    return Microbatch(lay(mb.ingress), tuple((lay(a), lay(m)) for a, m in mb.layers))


def _next_fit(order, lengths: dict, target: int, opening=()) -> tuple:
    """Samples in ``order`` cut into packs of at most ``target`` tokens (a pack always takes its
    first sample); each pack sorted; ``opening`` is an extra first pack."""
    packs = [tuple(sorted(opening))] if opening else []
    pack, tokens = [], 0
    for s in order:
        if pack and tokens + lengths[s] > target:
            packs.append(tuple(sorted(pack)))
            pack, tokens = [], 0
        pack.append(s)
        tokens += lengths[s]
    if pack:
        packs.append(tuple(sorted(pack)))
    return tuple(packs)


# ------------------------------------------------------------------ pool packing proposals
def _memory_targets(search: "_Search") -> list[int]:
    """Token targets per microbatch from the saved-activation headroom (search seeds only,
    never an admission rule): 0.5/0.8/1.0/1.3 of the nominal capacity, also rounded down to
    a multiple of world * gcd(lengths), never below the longest sample."""
    m, lengths, world = search.model, search.lengths, search.world
    base = Evaluator(m, lengths, world, search.pattern).base
    h, f, d = m.hidden, m.ffn, m.gdn_heads * m.gdn_dim
    per_token = 4 * h + len(search.pattern) * 2 * (12 * h + 3 * f + max(5 * d, h + 2 * m.kv_heads * m.head_dim))
    nominal = max(1, int((m.budget - base) / per_token)) * world
    longest = max(lengths.values())
    targets = {max(longest, int(nominal * scale)) for scale in (0.5, 0.8, 1.0, 1.3)}
    quantum = world * math.gcd(*lengths.values())
    targets |= {max(longest, t // quantum * quantum) for t in tuple(targets)}
    return sorted(targets)


def _plain_proposals(lengths, targets):
    for order in (sorted(lengths), sorted(lengths, key=lambda s: (-lengths[s], s))):
        for target in targets:
            yield _next_fit(order, lengths, target)


def _homogeneous_proposals(lengths, targets):
    """Samples of one length together, longest lengths first, ``target // length`` per pack."""
    by_length: dict[int, list[int]] = {}
    for s in sorted(lengths):
        by_length.setdefault(lengths[s], []).append(s)
    for target in targets:
        packs = []
        for n, samples in sorted(by_length.items(), reverse=True):
            step = max(1, target // n)
            packs += [tuple(samples[i:i + step]) for i in range(0, len(samples), step)]
        yield tuple(packs)


def _balanced_proposals(lengths, world, targets):
    """The heaviest sample at CP p paired with short samples worth about (world - p) / p times
    its tokens (equal linear work on the CP1 ranks), the rest packed to each target."""
    order = sorted(lengths, key=lambda s: (-lengths[s], s))
    anchor = order[0]
    shortest_first = sorted(order[1:], key=lambda s: (lengths[s], s))
    width = world // 2
    while width:
        if width == 1 or lengths[anchor] % (2 * width) == 0:
            goal = lengths[anchor] * (world - width) / width
            partners, tokens = [], 0
            for s in shortest_first:
                if tokens + lengths[s] <= goal:
                    partners.append(s)
                    tokens += lengths[s]
            if len(partners) >= world - width:
                paired = frozenset((anchor, *partners))
                rest = [s for s in order if s not in paired]
                for target in targets:
                    yield _next_fit(rest, lengths, target, opening=paired)
        width //= 2


def _heavy_tail_proposals(search: "_Search", targets):
    """Several numbers of large samples (>= half the longest) per microbatch, each block topped up
    with 0, 1, 2, 4, ... of the shortest samples, the remaining short pool packed to each target."""
    lengths, m = search.lengths, search.model
    ceiling = m.token_capacity_upper_bound(search.pattern, search.world)
    largest, smallest = max(lengths.values()), min(lengths.values())
    heavy = sorted((s for s in lengths if lengths[s] >= largest / 2), key=lambda s: (-lengths[s], s))
    chosen = set(heavy)
    tail = sorted((s for s in lengths if s not in chosen), key=lambda s: (lengths[s], s))
    if not tail or largest < 4 * smallest:
        return
    for count in range(1, min(len(heavy), search.world // m.ranks_per_node, ceiling // largest) + 1):
        blocks = [heavy[i:i + count] for i in range(0, len(heavy), count)]
        for extra in sorted({0, 1, 2, 4, 8, 16, 32, len(tail) // len(blocks)}):
            for target in targets:
                packs, cursor = [], 0
                for block in blocks:
                    pack, total = list(block), sum(lengths[s] for s in block)
                    while len(pack) - len(block) < extra and cursor < len(tail) \
                            and total + lengths[tail[cursor]] <= ceiling:
                        pack.append(tail[cursor])
                        total += lengths[tail[cursor]]
                        cursor += 1
                    packs.append(tuple(sorted(pack)))
                yield tuple(packs) + _next_fit(tail[cursor:], lengths, target)


# ------------------------------------------------------------------ the search
class _Search:
    def __init__(self, lengths, world, pattern, model, options):
        self.lengths, self.world, self.pattern = lengths, world, pattern
        self.model, self.options = model, options
        self.states = 0
        self.truncated = False
        self.cache: dict = {}
        self.incumbent = None
        self.packings_examined = 0

    def count_state(self) -> None:
        self.states += 1
        if self.states > self.options.max_states:
            raise SearchLimit("Search state budget exhausted; no global optimum is certified")

    def batch(self, ids):
        """Best (cost, microbatch) of these samples, solved once per length shape (sample ids are
        restored after solving; no content hashes are involved)."""
        ids = tuple(sorted(ids))
        shape = tuple(self.lengths[i] for i in ids)
        if shape not in self.cache:
            local = dict(enumerate(shape))
            fits = sum(shape) <= self.model.token_capacity_upper_bound(self.pattern, self.world)
            self.cache[shape] = _PathSearch(self, local).run() if fits else None
        answer = self.cache[shape]
        return None if answer is None else (answer[0], _relabel(answer[1], ids))

    def exact(self):
        ids = tuple(sorted(self.lengths))

        @lru_cache(None)
        def best_cover(mask: int):
            """Cheapest packing of the samples in ``mask``: the pack holding the lowest sample is
            chosen among every subset containing it, largest bitmask first."""
            if not mask:
                return 0.0, ()
            lowest, best = mask & -mask, None
            sub = mask
            while sub:
                if sub & lowest:
                    head = self.batch(tuple(ids[i] for i in range(len(ids)) if sub >> i & 1))
                    rest = best_cover(mask ^ sub) if head is not None else None
                    if rest is not None and (best is None or head[0] + rest[0] < best[0]):
                        best = (head[0] + rest[0], (head[1],) + rest[1])
                sub = (sub - 1) & mask
            return best

        return best_cover((1 << len(ids)) - 1)

    def proposals(self) -> list[tuple]:
        targets = _memory_targets(self)
        out = list(_plain_proposals(self.lengths, targets))
        if self.options.homogeneous_packing:
            out += _homogeneous_proposals(self.lengths, targets)
        if self.options.balanced_packing:
            # the known coverage correction goes first so that it survives tight budgets
            out = list(_balanced_proposals(self.lengths, self.world, targets)) + out
        if self.options.heavy_tail_packing:
            out = list(_heavy_tail_proposals(self, targets)) + out
        return out

    def bounded(self):
        seen, best = set(), None
        for packing in self.proposals():
            if packing in seen:
                continue
            seen.add(packing)
            self.packings_examined += 1
            rows = []
            for ids in packing:
                row = self.batch(ids)
                if row is None:
                    break
                rows.append(row)
            else:
                total = sum(r[0] for r in rows)
                if best is None or total < best[0]:
                    best = self.incumbent = (total, tuple(r[1] for r in rows))
        return best


DOMAIN = ("aligned dyadic groups; ascending sample order per pack; all ranks nonempty; no padding; fixed G/* kernel "
          "modes; independent MLP placement")
OBJECTIVE = ("minimize allocated GPU-ms for fixed useful input work; fixed world makes this equivalent to sum complete "
             "F+B microbatch times plus update/sync; all allocated ranks and idle waits counted")


def _score(plan: Plan, lengths, model):
    evidence = [Evaluator(model, lengths, plan.world, plan.pattern).evaluate(b) for b in plan.microbatches]
    return sum(row["predicted_ms"] for row in evidence) + model.update_ms, evidence


def solve(lengths: dict, world: int, pattern: str, model, options: SearchOptions = SearchOptions()) -> dict:
    bad_lengths = any(type(s) is not int or type(n) is not int or n <= 0 for s, n in lengths.items())
    if not lengths or world <= 0 or world & (world - 1) or not pattern or set(pattern) - set("G*") or bad_lengths:
        raise ValueError("Invalid lengths, world or pattern")
    if options.mode == "exact" and (len(lengths) > 6 or world > 4):
        raise ValueError("Exact domain is limited to <=6 samples and <=4 ranks; use bounded mode")
    if getattr(model, "recompute_tokens", None) is not None:
        # the search prices a microbatch layer by layer; whether it recomputes depends on all of its
        # layouts at once, which the incremental objective cannot see
        raise ValueError("The joint solver prices microbatches without recompute; pass a model with "
                         "recompute_tokens=None (the online selector handles recompute)")
    search = _Search(lengths, world, pattern, model, options)
    limit_hit = False
    try:
        answer = search.exact() if options.mode == "exact" else search.bounded()
    except SearchLimit:
        if options.mode == "exact":
            raise
        limit_hit, answer = True, search.incumbent
    meta = {"search_mode": options.mode, "states_examined": search.states, "state_budget_exhausted": limit_hit,
            "pool_packings_examined": search.packings_examined, "microbatch_shapes_solved": len(search.cache),
            "beam_pruned": search.truncated, "domain": DOMAIN, "objective": OBJECTIVE,
            "model_provenance": model.provenance, "gpu_admitted": False,
            "max_attention_cp": options.max_attention_cp}
    if answer is None:
        status = ("search_budget_exhausted" if limit_hit else
                  "infeasible_in_declared_domain" if options.mode == "exact" else "no_feasible_plan_found")
        return {**meta, "status": status, "plan": None}
    plan = Plan(world, pattern, answer[1])
    validate_plan(plan, lengths)
    predicted, evidence = _score(plan, lengths, model)
    if not all(row["fits"] for row in evidence):
        raise AssertionError("Solver and full-plan memory accounting disagree")
    if not math.isclose(predicted, answer[0] + model.update_ms, rel_tol=1e-10, abs_tol=1e-8):
        raise AssertionError("Solver and full-plan objective disagree")
    if options.mode == "bounded":
        plan, meta["memory_selection"] = prefer_lower_memory(plan, lengths, model, options.memory_time_tolerance)
        validate_plan(plan, lengths)
        predicted, evidence = _score(plan, lengths, model)
        meta["objective"] += "; bounded CP1 memory tie-break within declared time tolerance"
    status = "optimal_in_declared_domain" if options.mode == "exact" else "best_found_no_optimality_certificate"
    return {**meta, "status": status, "plan": plan.to_dict(), "predicted_update_ms": predicted,
            "resource_metrics": resource_metrics(lengths, world, pattern, model, predicted),
            "cp_response_evidence": response_coverage(plan, lengths, model), "budget_bytes": model.budget,
            "microbatch_evidence": evidence}
