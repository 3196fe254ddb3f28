"""Tracing and profiling hooks: NVTX ranges, a profiler capture window, and a
per-kernel device-time breakdown of one training step.

* ``nvtx(name)`` is a context manager that opens an NVTX range when ranges are
  enabled (``enable_nvtx(True)``, the launcher's ``--nvtx-ranges`` or
  ``PRISM_NVTX=1``) and costs one attribute test otherwise. The executor marks
  every microbatch, layer and CP-transition route, so an ``nsys`` timeline
  groups kernels by layer and microbatch (the reference marks the same units
  with NVTX for its nsys wrapper: scripts/run_manual_gdn_cp_case.sh:284-310,
  SD/runtime.py:93-95).
* ``ProfileWindow(start, end, ranks)`` calls ``cudaProfilerStart`` before step
  ``start`` and ``cudaProfilerStop`` after step ``end`` on the listed ranks, for
  ``nsys --capture-range cudaProfilerApi`` or ``ncu --profile-from-start off``
  (the launcher's ``--profile --profile-step-start/end --profile-ranks``).
* ``python -m prism_cp_b200.utils.tracing --model hybrid-1.3b --seq-len 32768``
  runs warm-up steps of the model on one GPU and prints the device time of
  every kernel of one step (``torch.profiler`` CUDA activity), sorted by total
  time: the per-kernel share table a roofline analysis starts from.
"""

from __future__ import annotations

import argparse
import contextlib
import os
import sys

import torch

_NVTX = os.environ.get("PRISM_NVTX", "0") == "1"


def enable_nvtx(on: bool = True) -> None:
    global _NVTX
    _NVTX = bool(on)


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def _range(name: str):
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx(name: str):
    """An NVTX range around a block when ranges are enabled (CUDA builds only)."""
    if _NVTX and torch.cuda.is_available():
        return _range(name)
    return contextlib.nullcontext()


class ProfileWindow:
    """Start the CUDA profiler API capture before step ``start``, stop it after step ``end``."""

    def __init__(self, start: int, end: int, ranks=(0,), rank: int = 0, enabled: bool = True):
        if end < start:
            raise ValueError("profile window ends before it starts")
        self.start, self.end = start, end
        self.active = enabled and (not ranks or rank in ranks) and torch.cuda.is_available()
        self.running = False

    def before(self, step: int) -> None:
        if self.active and step == self.start and not self.running:
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            self.running = True

    def after(self, step: int) -> None:
        if self.running and step == self.end:
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            self.running = False


def step_breakdown(model_name: str = "hybrid-1.3b", seq_len: int = 32768, seqs: int = 1, warmup: int = 2,
                   rows: int = 45) -> str:
    """Per-kernel device-time table of one training step on ``cuda:0`` (single GPU, CP=1)."""
    from torch.profiler import ProfilerActivity, profile

    from ..models.config import PRESETS
    from ..models.hybrid import HybridModel
    from ..parallel.teams import Teams
    from ..planner.fixed import uniform_plan
    from ..runtime.batch import make_batch
    from ..runtime.trainer import Trainer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS[model_name]()
    model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)
    trainer = Trainer(model, Teams(1), dev)
    batch = make_batch([seq_len] * seqs, cfg.vocab_size, seed=1, pin=True)
    plan = uniform_plan(batch.lengths, 1, 1, seq_len, cfg.pattern)
    inputs = [h.to(dev) for h in trainer.prepare(batch, plan)]
    for _ in range(warmup):
        trainer.train_step(batch, plan, inputs, read_loss=False)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.train_step(batch, plan, inputs, read_loss=False)
        torch.cuda.synchronize()
    from ..ops._lib import check_status
    check_status(dev)
    return prof.key_averages().table(sort_by="cuda_time_total", row_limit=rows, max_name_column_width=90)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="per-kernel device time of one training step")
    ap.add_argument("--model", default="hybrid-1.3b")
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--seqs", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rows", type=int, default=45)
    ap.add_argument("--output", default=None)
    args = ap.parse_args(argv)
    table = step_breakdown(args.model, args.seq_len, args.seqs, args.warmup, args.rows)
    if args.output:
        with open(args.output, "w") as f:
            f.write(table)
    print(table)
    return 0


if __name__ == "__main__":
    sys.exit(main())
