#!/usr/bin/env python
"""Training throughput benchmark of the hybrid GDN:GQA decoder.

Default workload: the 1.3B hybrid (24 layers, 18 GDN + 6 GQA, hidden 2048,
vocab 32000), bf16, one global batch of 1M tokens of variable-length
documents (lengths log-normal with median 4K, clipped to 512..128K, seeded,
multiples of 16 tokens so the same batch runs at every N; synthetic token ids
uniform over the vocabulary, random-init weights). The online planner picks
the CP degree of the GDN and of the GQA layers for the batch on N GPUs from
the calibrated B200 cost model and packs the documents into microbatches;
a microbatch that holds more than 32K tokens on a rank (a document too long
for its team) recomputes its layers in the backward. Gradient reduce-scatter
overlaps the last backward and the parameter all-gather the next forward
(``--no-overlap``: both after the step). ``--workload fixed --plan uniform``
runs 8 documents x 32768 tokens at CP = N instead.

Measured: W warm-up steps, then exactly K steps between barrier +
synchronize, timed with CUDA events on the launching stream, max over ranks.
Each step's working set (activations of 32K-token microbatches, ~GBs) is far
larger than the 126 MB L2. A second loop times the same K steps end to end
through the public ``Trainer.train_step`` API with the inputs copied from
pinned host memory every step and the loss read back to the host.
Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "train tokens/s (device-timed, max over ranks) on var-len batches at 1/2/4/8 B200"


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--model", default="hybrid-1.3b")
    ap.add_argument("--workload", choices=("fixed", "lognormal"), default="lognormal")
    ap.add_argument("--plan", choices=("uniform", "online"), default="online",
                    help="uniform: CP = N for every layer; online: per-batch (cp_gdn, cp_gqa) from the "
                         "calibrated B200 cost model")
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--tokens-per-rank", type=int, default=32768)
    ap.add_argument("--total-tokens", type=int, default=1 << 20)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="reduce-scatter the gradients after the backward and all-gather the parameters after the "
                         "update on the compute stream (default: both bucketed on side streams, overlapping the "
                         "last backward and the next forward)")
    ap.add_argument("--recompute-tokens", type=int, default=32768,
                    help="microbatches with more tokens than this on a rank recompute their layers in the backward "
                         "(0: never)")
    return ap.parse_args()


REFERENCE_UNAVAILABLE = (
    "the reference is a research harness over an unmounted Megatron-LM fork (no setup.py/pyproject, "
    "pip install fails; its GPU path imports megatron.core, TransformerEngine and FLA, none of which exist here)")


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [x.strip() for x in line.split(",")]))

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.__exit__()
        t0, t1 = getattr(self, "t0", 0.0), getattr(self, "t1", float("inf"))
        window = [r for t, r in self.rows if t0 <= t <= t1]
        self.rows = window or [r for _, r in self.rows]
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in self.rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def progress(rank: int, msg: str) -> None:
    """Phase markers on stderr (stdout carries only the JSON line)."""
    if rank == 0:
        print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": REFERENCE_UNAVAILABLE}))
        return 0

    import datetime
    import torch
    import torch.distributed as dist

    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.runtime.trainer import Trainer
    from prism_cp_b200.runtime.workload import build as build_workload

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=600))
    cfg = PRESETS[args.model]()
    try:
        wl = build_workload(cfg, world, args.workload, args.plan, seqs=args.seqs, seq_len=args.seq_len,
                            tokens_per_rank=args.tokens_per_rank, total_tokens=args.total_tokens, seed=args.seed,
                            recompute_tokens=args.recompute_tokens or None)
    except ValueError as err:
        raise SystemExit(f"--plan {args.plan}: {err}")
    batch, plan, workload, plan_desc, predicted_ms = wl.batch, wl.plan, wl.description, wl.parallelism, \
        wl.predicted_ms

    model = HybridModel(cfg, dtype=torch.bfloat16, device=device, seed=0)
    teams = Teams(world)
    trainer = Trainer(model, teams, device, overlap_grad_reduce=not args.no_overlap,
                      overlap_param_gather=not args.no_overlap, recompute_tokens=args.recompute_tokens or None)
    host_inputs = trainer.prepare(batch, plan, pin=True)
    dev_inputs = [h.to(device) for h in host_inputs]
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    progress(rank, f"model ready ({cfg.parameter_count() / 1e9:.2f}B params, {len(plan.microbatches)} microbatches)")
    # the clock sampler's process starts before any GPU work, its samples are cut to the timed region
    clocks = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        trainer.train_step(batch, plan, dev_inputs, read_loss=False)
    progress(rank, "warm-up done")
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    start.record()
    for i in range(args.steps):
        trainer.train_step(batch, plan, dev_inputs, read_loss=False)
        progress(rank, f"timed step {i + 1}/{args.steps} queued")
    end.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    barrier()
    torch.cuda.synchronize()
    ms = torch.tensor([start.elapsed_time(end) / args.steps], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_step = float(ms.item())
    tokens = batch.total_tokens
    value = tokens / (ms_step / 1000.0)

    progress(rank, f"timed loop: {ms_step:.1f} ms/step")
    e2e = None
    if not args.no_e2e:
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            res = trainer.train_step(batch, plan, host_inputs, read_loss=True)
        torch.cuda.synchronize()
        barrier()
        dt = torch.tensor([(time.perf_counter() - t0) / args.steps], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        h2d = sum(h.nbytes for h in host_inputs)
        e2e = {"value": tokens / float(dt.item()), "unit": "tokens/s", "ms_per_step": 1000 * float(dt.item()),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "loss": res.loss,
               "api": "prism_cp_b200.runtime.trainer.Trainer.train_step"}

    progress(rank, "end-to-end loop done")
    launches = count_launches(trainer, batch, plan, dev_inputs)
    mem_peak = torch.cuda.max_memory_allocated(device)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids, random-init weights)",
            "config": dict(model=f"{cfg.name} ({cfg.num_layers}L {cfg.pattern.count('G')} GDN + "
                                 f"{cfg.pattern.count('*')} GQA, h{cfg.hidden_size}, "
                                 f"{cfg.parameter_count() / 1e9:.2f}B params)",
                           parallelism=plan_desc, workload=args.workload, microbatches=len(plan.microbatches),
                           planner_predicted_ms_per_step=predicted_ms, recompute_tokens=args.recompute_tokens,
                           grad_sync="serial" if args.no_overlap else
                           "overlapped (reduce-scatter in the last backward, all-gather in the next forward)",
                           l2="per-step working set (32K-token activations) far exceeds the 126 MB L2",
                           **workload),
            "clocks": clocks.summary(), "e2e": e2e, "gpu_launches": launches * args.steps,
            "peak_allocated_gib": round(mem_peak / 2 ** 30, 2),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def count_launches(trainer, batch, plan, inputs) -> int:
    """Kernels of this repo's library launched by one step (counted on an extra, untimed step)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.train_step(batch, plan, inputs, read_loss=False)
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        if ev.device_type is not None and "cuda" in str(ev.device_type).lower() and "prism" in ev.name:
            n += 1
    return n


if __name__ == "__main__":
    sys.exit(main())
