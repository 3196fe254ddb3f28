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
    def __init__(self, world: int | None = None, backend: str | None = None):
        self.initialized = dist.is_available() and dist.is_initialized()
        self.world = world if world is not None else (dist.get_world_size() if self.initialized else 1)
        self.rank = dist.get_rank() if self.initialized else 0
        self.groups: dict[tuple[int, ...], object] = {}
        if self.initialized and self.world > 1:
            for ranks in dyadic_intervals(self.world):
                if len(ranks) == self.world:
                    group = dist.group.WORLD
                elif len(ranks) == 1:
                    group = None
                else:
                    group = dist.new_group(list(ranks), backend=backend)
                if self.rank in ranks:
                    self.groups[ranks] = group

    def team(self, ranks: tuple[int, ...]):
        if len(ranks) == 1:
            return None
        if ranks not in self.groups:
            raise KeyError(f"rank {self.rank} is not a member of team {ranks}")
        return self.groups[ranks]

    @property
    def world_group(self):
        return dist.group.WORLD if self.initialized else None
