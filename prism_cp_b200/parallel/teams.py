"""Pre-created CP teams: one process group per aligned dyadic rank interval.

For a world of W ranks there are 2W - 1 such intervals (15 on 8 GPUs). They
are created once at start-up in a fixed order on every rank (every rank takes
part in every ``new_group`` call, as torch.distributed requires), so the
planner can choose a different CP degree for every layer and microbatch
without re-initialising anything (reference: joint_cp/adapter.py:83-99).
"""

from __future__ import annotations

import torch.distributed as dist


def dyadic_intervals(world: int) -> list[tuple[int, ...]]:
    out = []
    width = world
    while width >= 1:
        for start in range(0, world, width):
            out.append(tuple(range(start, start + width)))
        width //= 2
    return sorted(out, key=lambda r: (len(r), r))


class Teams:
    """Dyadic CP teams over logical ranks.

    Without tensor parallelism a logical rank is a global rank. With a
    ``TPContext`` of size tp, logical rank l of TP index i is global rank
    l * tp + i; every TP index gets its own teams (all ranks take part in all
    ``new_group`` calls) and this rank keeps the teams of its own index.
    """

    def __init__(self, world: int | None = None, backend: str | None = None, tp=None):
        self.initialized = dist.is_available() and dist.is_initialized()
        tp_on = tp is not None and tp.enabled
        if tp_on:
            self.world, self.rank = tp.logical_world, tp.logical_rank
            self.rank_map = tp.rank_map()
            indices = range(tp.tp)
        else:
            self.world = world if world is not None else (dist.get_world_size() if self.initialized else 1)
            self.rank = dist.get_rank() if self.initialized else 0
            self.rank_map = list(range(self.world))
            indices = [0]
        self.groups: dict[tuple[int, ...], object] = {}
        self._world_group = dist.group.WORLD if (self.initialized and not tp_on) else None
        if self.initialized and self.world > 1:
            for ranks in dyadic_intervals(self.world):
                for index in indices:
                    members = [l * tp.tp + index for l in ranks] if tp_on else list(ranks)
                    if len(ranks) == 1:
                        group = None
                    elif len(ranks) == self.world and not tp_on:
                        group = dist.group.WORLD
                    else:
                        group = dist.new_group(members, backend=backend)
                    mine = (not tp_on or index == tp.index) and self.rank in ranks
                    if mine:
                        self.groups[ranks] = group
                        if len(ranks) == self.world:
                            self._world_group = group

    def team(self, ranks: tuple[int, ...]):
        if len(ranks) == 1:
            return None
        if ranks not in self.groups:
            raise KeyError(f"rank {self.rank} is not a member of team {ranks}")
        return self.groups[ranks]

    def global_rank(self, logical: int) -> int:
        return self.rank_map[logical]

    @property
    def world_group(self):
        """Group of all logical ranks of this rank's TP index (the whole world without TP)."""
        return self._world_group
