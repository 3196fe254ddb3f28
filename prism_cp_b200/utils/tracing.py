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
* ``torchrun --nproc-per-node N -m prism_cp_b200.utils.tracing --distributed``
  does the same on N ranks at CP = N and reduces every rank's kernel timeline
  to categories (attention, GDN, GEMM, NCCL, P2P, ...), the step's device time
  (CUDA events, max over ranks), the busy time (union of kernel intervals),
  the communication time not hidden under compute, and the idle time: the
  table that says which kernel or collective holds a multi-GPU step above
  linear scaling.
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


# kernel-name patterns of each category (first match wins); NCCL and P2P are communication
CATEGORIES = (
    ("nccl", ("nccl",)),
    ("p2p", ("symm::", "gather_rows", "signal_all", "wait_all", "attention_peer", "_peer")),
    ("attention", ("attn",)),
    ("gdn", ("gdn", "conv_", "l2norm")),
    ("gemm", ("gemm",)),
    ("norm/act/optim", ("rownorm", "swiglu", "rope", "adamw", "sumsq", "column_sum", "cross_entropy", "ce_")),
    ("copy", ("memcpy", "memset", "copy", "cat", "index")),
)
COMM = ("nccl", "p2p")


def categorize(name: str) -> str:
    low = name.lower()
    for cat, keys in CATEGORIES:
        if any(k in low for k in keys):
            return cat
    return "other"


def _union(intervals):
    """Total length of the union of [start, end) intervals, and the merged list."""
    merged = []
    for a, b in sorted(intervals):
        if merged and a <= merged[-1][1]:
            merged[-1][1] = max(merged[-1][1], b)
        else:
            merged.append([a, b])
    return sum(b - a for a, b in merged), merged


def _overlap(merged_a, merged_b) -> float:
    """Length of the intersection of two merged interval lists."""
    i = j = 0
    total = 0.0
    while i < len(merged_a) and j < len(merged_b):
        a0, a1 = merged_a[i]
        b0, b1 = merged_b[j]
        lo, hi = max(a0, b0), min(a1, b1)
        if hi > lo:
            total += hi - lo
        if a1 < b1:
            i += 1
        else:
            j += 1
    return total


def timeline_summary(kernels, step_ms: float) -> dict:
    """Reduce one rank's kernels ``[(name, start_us, end_us)]`` of one step to category totals,
    busy time (union), communication not overlapped by compute, and idle time (all in ms)."""
    cats: dict = {}
    comm, compute, every = [], [], []
    for name, a, b in kernels:
        c = categorize(name)
        cats[c] = cats.get(c, 0.0) + (b - a) / 1000.0
        (comm if c in COMM else compute).append((a, b))
        every.append((a, b))
    busy, _ = _union(every)
    comm_len, comm_m = _union(comm)
    _, comp_m = _union(compute)
    exposed = comm_len - _overlap(comm_m, comp_m)
    span = (max(b for _, _, b in kernels) - min(a for _, a, _ in kernels)) / 1000.0 if kernels else 0.0
    return dict(step_ms=step_ms, span_ms=span, busy_ms=busy / 1000.0, exposed_comm_ms=exposed / 1000.0,
                idle_ms=max(0.0, span - busy / 1000.0), categories=cats)


def _kernels_of(prof):
    out = []
    for ev in prof.events():
        if ev.device_type is not None and "cuda" in str(ev.device_type).lower():
            out.append((ev.name, float(ev.time_range.start), float(ev.time_range.end)))
    return out


def distributed_breakdown(model_name: str, seqs: int, seq_len: int, tokens_per_rank: int, warmup: int,
                          timed: int, top: int = 12, workload: str = "fixed", plan_kind: str = "uniform",
                          recompute_tokens: int | None = 32768) -> str | None:
    """Per-rank category breakdown of one training step of a benchmark workload (torchrun ranks,
    NCCL); returns the markdown report on rank 0, None elsewhere."""
    import datetime
    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile

    from ..models.config import PRESETS
    from ..models.hybrid import HybridModel
    from ..parallel.teams import Teams
    from ..runtime.trainer import Trainer
    from ..runtime.workload import build

    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    rank = dist.get_rank() if world > 1 else 0
    cfg = PRESETS[model_name]()
    model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)
    trainer = Trainer(model, Teams(world), dev, recompute_tokens=recompute_tokens)
    wl = build(cfg, world, workload, plan_kind, seqs=seqs, seq_len=seq_len, tokens_per_rank=tokens_per_rank,
               recompute_tokens=recompute_tokens)
    batch, plan = wl.batch, wl.plan
    inputs = [h.to(dev) for h in trainer.prepare(batch, plan)]
    for _ in range(warmup):
        trainer.train_step(batch, plan, inputs, read_loss=False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(timed):
        trainer.train_step(batch, plan, inputs, read_loss=False)
    end.record()
    torch.cuda.synchronize()
    step = torch.tensor([start.elapsed_time(end) / timed], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(step, op=dist.ReduceOp.MAX)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.train_step(batch, plan, inputs, read_loss=False)
        torch.cuda.synchronize()
    from ..ops._lib import check_status
    check_status(dev)
    kernels = _kernels_of(prof)
    summary = timeline_summary(kernels, float(step.item()))
    per_kernel: dict = {}
    for name, a, b in kernels:
        per_kernel[name] = per_kernel.get(name, 0.0) + (b - a) / 1000.0
    summary["top"] = sorted(per_kernel.items(), key=lambda kv: -kv[1])[:top]
    gathered = [None] * world
    if world > 1:
        dist.all_gather_object(gathered, summary)
        dist.barrier()
        dist.destroy_process_group()
    else:
        gathered = [summary]
    if rank != 0:
        return None
    return format_breakdown(gathered, dict(model=model_name, seqs=len(batch.lengths),
                                           seq_len=max(batch.lengths.values()), world=world, impl=os.environ.get("PRISM_CP_ATTENTION", "peer"),
                                           plan=wl.parallelism, workload=workload))


def format_breakdown(ranks: list, meta: dict) -> str:
    cats = sorted({c for r in ranks for c in r["categories"]})
    lines = [f"step breakdown: {meta['model']}, {meta.get('workload', 'fixed')} workload, {meta['seqs']} documents "
             f"(longest {meta['seq_len']} tokens), plan {meta.get('plan', 'cp%d' % meta['world'])} on "
             f"{meta['world']} GPU(s), CP attention {meta['impl']} where the layout allows it",
             f"device step time (CUDA events, max over ranks): {ranks[0]['step_ms']:.1f} ms", "",
             "| rank | span ms | busy ms | idle ms | comm not under compute ms | " + " | ".join(cats) + " |",
             "|" + "---|" * (5 + len(cats))]
    for i, r in enumerate(ranks):
        vals = " | ".join(f"{r['categories'].get(c, 0.0):.1f}" for c in cats)
        lines.append(f"| {i} | {r['span_ms']:.1f} | {r['busy_ms']:.1f} | {r['idle_ms']:.1f} | "
                     f"{r['exposed_comm_ms']:.1f} | {vals} |")
    worst = max(range(len(ranks)), key=lambda i: ranks[i]["span_ms"])
    lines += ["", f"top kernels of rank {worst} (device ms):", ""]
    lines += [f"| {ms:.2f} | `{name[:100]}` |" for name, ms in ranks[worst]["top"]]
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="per-kernel device time of one training step")
    ap.add_argument("--model", default="hybrid-1.3b")
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--seqs", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rows", type=int, default=45)
    ap.add_argument("--output", default=None)
    ap.add_argument("--distributed", action="store_true",
                    help="CP = world over torchrun ranks: per-rank categories, exposed communication, idle time")
    ap.add_argument("--tokens-per-rank", type=int, default=32768)
    ap.add_argument("--timed", type=int, default=2)
    ap.add_argument("--workload", choices=("fixed", "lognormal"), default="fixed",
                    help="with --distributed: the benchmark workload to break down")
    ap.add_argument("--plan", choices=("uniform", "online"), default="uniform")
    args = ap.parse_args(argv)
    if args.distributed:
        report = distributed_breakdown(args.model, args.seqs, args.seq_len, args.tokens_per_rank, args.warmup,
                                       args.timed, workload=args.workload, plan_kind=args.plan)
        if report is not None:
            if args.output:
                with open(args.output, "w") as f:
                    f.write(report + "\n")
            print(report)
        return 0
    table = step_breakdown(args.model, args.seq_len, args.seqs, args.warmup, args.rows)
    if args.output:
        with open(args.output, "w") as f:
            f.write(table)
    print(table)
    return 0


if __name__ == "__main__":
    sys.exit(main())
