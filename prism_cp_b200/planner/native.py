"""Native N: the dynamic-CP greedy scheduler the reference compares against.

The reference replays Megatron's ``next_hdp_group_packing_aware`` by compiling
it from an external Megatron source tree (experiments/sequence_dynamic_cp/
native.py:14-86). That tree is not available, so this is a re-derivation of its
documented behaviour - workload ``(L^2 + beta L) / cp``, minimum CP, greedy fill
with tie-breaks, per-rank token capacity ``K`` - checked against the frozen
``rank_ids`` it produced (golden plans from the reference's results), its two
unit regressions and its square-vs-hybrid counterexample (the square workload
packs short samples to the token capacity and the idle ranks then double the
long sample's group; a token-weighted workload spreads them):

one microbatch (``next_group``):
  1. samples are visited in descending workload order (ties: input order);
  2. a sample needs ``cp = max(min_cp, 2^ceil(log2(L / K)))`` ranks;
  3. the candidate group is the least-loaded existing group (ties: lowest start)
     whose per-rank tokens stay <= K, whose per-rank workload stays within
     ``(local_tall + beta) * K * (1 + DELTA)`` (``local_tall`` = longest sample
     of the microbatch) and that divides the sample by 2*cp;
  4. the sample joins it when that does not raise the heaviest group's workload
     (it fills the room the tallest sample leaves); otherwise it opens a new
     group on the first aligned block of ``cp`` idle ranks; with no idle block
     it joins the candidate anyway; with no candidate it is left over;
  5. idle ranks are filled by doubling the smallest group (lowest start first)
     and shifting later groups right; when a world is not a power of two, or no
     doubling fits, all samples of the microbatch become one world-wide group.

``replay`` repeats ``next_group`` until every sample is consumed and returns
``rank_ids`` per microbatch (each rank's sample list), the executor format.
"""

from __future__ import annotations

import math

DYNAMIC_CP_WORKLOAD_CAP_DELTA = 0.0


def gpus_needed(length: int, cap: int, min_cp: int = 1) -> int:
    need = max(1, math.ceil(length / cap))
    return max(min_cp, 1 << (need - 1).bit_length())


def _aligned_free(free: list[bool], size: int):
    for start in range(0, len(free) - size + 1, size):
        if all(free[start:start + size]):
            return start
    return None


def _fill_idle(groups: list[dict], world: int) -> list[dict]:
    used = sum(g["size"] for g in groups)
    if used == world:
        return groups
    if world & (world - 1):
        merged = [s for g in groups for s in g["samples"]]
        return [{"start": 0, "size": world, "samples": merged}]
    groups = sorted(groups, key=lambda g: g["start"])
    while sum(g["size"] for g in groups) < world:
        smallest = min(g["size"] for g in groups)
        target = next(g for g in groups if g["size"] == smallest)
        target["size"] *= 2
        # re-pack starts left to right; keep every group aligned to its size
        pos = 0
        ok = True
        for g in groups:
            if pos % g["size"]:
                pos += g["size"] - pos % g["size"]
            g["start"] = pos
            pos += g["size"]
            if pos > world:
                ok = False
        if not ok:
            merged = [s for g in groups for s in g["samples"]]
            return [{"start": 0, "size": world, "samples": merged}]
    return groups


def next_group(remaining: list[tuple[int, int]], world: int, cap: int, min_cp: int = 1, beta_tokens: float = 0.0):
    """One microbatch: returns (rank_ids, leftovers) for (sample_id, length) pairs."""
    if not remaining:
        return [[] for _ in range(world)], []
    order = sorted(range(len(remaining)),
                   key=lambda i: (-(remaining[i][1] ** 2 + beta_tokens * remaining[i][1]), i))
    local_tall = max(L for _, L in remaining)
    limit = (local_tall + beta_tokens) * cap * (1.0 + DYNAMIC_CP_WORKLOAD_CAP_DELTA)
    free = [True] * world
    groups: list[dict] = []
    leftovers = []
    for i in order:
        sid, L = remaining[i]
        need = gpus_needed(L, cap, min_cp)
        if need > world:
            raise ValueError(f"sample {sid} of length {L} needs CP{need} > world {world}")
        work = L * L + beta_tokens * L
        best = None
        for g in groups:
            c = g["size"]
            if c > 1 and L % (2 * c):
                continue
            if g["tokens"] + L / c > cap:
                continue
            if g["load"] + work / c > limit * (1 + 1e-12):
                continue
            key = (g["load"], g["start"])
            if best is None or key < best[0]:
                best = (key, g)
        heaviest = max((g["load"] for g in groups), default=0.0)
        start = None
        if best is None or best[1]["load"] + work / best[1]["size"] > heaviest * (1 + 1e-12):
            start = _aligned_free(free, need)
        if start is not None:
            for r in range(start, start + need):
                free[r] = False
            groups.append({"start": start, "size": need, "samples": [sid], "tokens": L / need, "load": work / need})
            continue
        if best is None:
            leftovers.append((sid, L))
            continue
        g = best[1]
        g["samples"].append(sid)
        g["tokens"] += L / g["size"]
        g["load"] += work / g["size"]
    if not groups:
        raise ValueError("Native scheduler made no progress")
    groups = _fill_idle(groups, world)
    rank_ids: list[list[int]] = [[] for _ in range(world)]
    for g in groups:
        for r in range(g["start"], g["start"] + g["size"]):
            rank_ids[r] = list(g["samples"])
    position = {q[0]: k for k, q in enumerate(remaining)}
    leftovers.sort(key=lambda p: position[p[0]])
    return rank_ids, leftovers


def replay(samples: list[tuple[int, int]], world: int, cap: int, min_cp: int = 1,
           beta_tokens: float = 0.0) -> list[list[list[int]]]:
    """Every microbatch of a global batch; fails if an iteration consumes nothing."""
    if beta_tokens < 0:
        raise ValueError("beta must be nonnegative")
    remaining = sorted(samples, key=lambda p: p[1], reverse=True)
    batches = []
    while remaining:
        ranks, leftovers = next_group(remaining, world, cap, min_cp, beta_tokens)
        if len(leftovers) >= len(remaining):
            raise ValueError("Native scheduler made no progress")
        batches.append(ranks)
        remaining = leftovers
    return batches
