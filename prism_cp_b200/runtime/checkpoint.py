"""Sharded checkpoints in the ``torch.distributed.checkpoint`` (torch_dist) layout.

A checkpoint directory holds, via ``torch.distributed.checkpoint.save``:
  * ``model``     - the bf16 model state (replicated on every rank, written once);
  * ``optimizer`` - each rank's fp32 master / Adam shard, keyed by rank (and by
    pipeline stage) so a resume on the same world size restores it exactly;
  * ``meta``      - step, scheduler position, plan cursor and RNG states.
Reference: Megatron ``--ckpt-format torch_dist --save --save-interval``
(scripts/run_manual_gdn_cp_case.sh:379,395-397), which the reference exposes
but never exercises.
"""

from __future__ import annotations

from pathlib import Path

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp


def _keys(trainer) -> tuple[str, str]:
    """(model key prefix, optimizer / RNG shard name) of this rank.

    A pipeline stage holds only its own layers, numbered from 0 inside the stage, and its optimizer
    ranks count from 0 inside the stage; a tensor-parallel index holds its own weight shards under
    the layer names every index uses. Both are qualified (by stage, by TP index) so that all ranks
    of one run write disjoint entries of the same checkpoint."""
    opt = trainer.optimizer
    info = getattr(trainer, "info", None)
    if info is not None and getattr(info, "pp", 1) > 1:
        return f"stage{info.stage}.", f"stage{info.stage}_rank{opt.rank}"
    tp = getattr(trainer, "tp", None)
    if tp is not None and tp.enabled:
        # each tensor-parallel index holds its own shard of the weights under the same names
        return f"tp{tp.index}.", f"tp{tp.index}_rank{opt.rank}"
    return "", f"rank{opt.rank}"


def _state(trainer, plan_cursor: int) -> dict:
    opt = trainer.optimizer
    opt.wait_parameters()  # an overlapped all-gather may still be writing the parameters
    prefix, shard = _keys(trainer)
    return {"model": {prefix + k: v for k, v in trainer.model.state_dict().items()},
            "optimizer": {shard: {"master": opt.master, "m": opt.m, "v": opt.v}},
            "meta": {"step": torch.tensor(opt.step_count), "plan_cursor": torch.tensor(plan_cursor),
                     "world": torch.tensor(opt.world),
                     f"cpu_rng_{shard}": torch.get_rng_state()}}


def save(trainer, directory: str | Path, plan_cursor: int = 0) -> Path:
    path = Path(directory) / f"iter_{trainer.optimizer.step_count:07d}"
    dcp.save(_state(trainer, plan_cursor), checkpoint_id=str(path))
    if not dist.is_initialized() or dist.get_rank() == 0:
        (Path(directory) / "latest_checkpointed_iteration.txt").write_text(str(trainer.optimizer.step_count))
    return path


def latest(directory: str | Path) -> Path | None:
    marker = Path(directory) / "latest_checkpointed_iteration.txt"
    if not marker.exists():
        return None
    return Path(directory) / f"iter_{int(marker.read_text()):07d}"


def load(trainer, path: str | Path) -> int:
    """Restore model, this rank's optimizer shard and counters; returns the plan cursor."""
    state = _state(trainer, 0)
    dcp.load(state, checkpoint_id=str(path))
    opt = trainer.optimizer
    if int(state["meta"]["world"]) != opt.world:
        raise ValueError("checkpoint world size differs from the current run")
    prefix, shard = _keys(trainer)
    trainer.model.load_state_dict({k[len(prefix):]: v for k, v in state["model"].items()})
    saved = state["optimizer"][shard]
    opt.master.copy_(saved["master"])
    opt.m.copy_(saved["m"])
    opt.v.copy_(saved["v"])
    opt.step_count = int(state["meta"]["step"])
    trainer.step_index = opt.step_count
    torch.set_rng_state(state["meta"][f"cpu_rng_{shard}"])
    return int(state["meta"]["plan_cursor"])
