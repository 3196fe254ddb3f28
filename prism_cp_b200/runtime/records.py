"""Per-rank step records, their compressed form and the run summary.

Every rank appends one JSON line per complete update to
``<output>/steps_rank{R}.jsonl`` with the fields the reference's analysis
tools read (experiments/sequence_dynamic_cp/runtime.py:442-516): losses, grad
norm, step, rank-max and local elapsed ms, peak allocated/reserved bytes,
tokens, samples, microbatches, sync payloads, the HBM budget and admission,
forward/backward counts and finite flags. ``compress`` folds all ranks into
``steps_by_rank.json.gz`` and ``summarize_records`` classifies a run as
``complete`` / ``actual_memory_guard_rejected`` / ``training_contract_failed`` /
``incomplete`` with the mean rank-max update time over the measured steps
(same rules as experiments/sequence_dynamic_cp/results_io.py:16-56).
"""

from __future__ import annotations

import gzip
import json
from pathlib import Path


class StepRecorder:
    def __init__(self, output: str | Path, rank: int):
        self.path = Path(output) / f"steps_rank{rank}.jsonl"
        self.path.parent.mkdir(parents=True, exist_ok=True)

    def write(self, record: dict) -> None:
        with self.path.open("a") as f:
            f.write(json.dumps(record, sort_keys=True) + "\n")


class RunRecords:
    """The auxiliary per-run records beside ``steps_rank*.jsonl``.

    * ``model_inventory.json`` (rank 0, once): every parameter's name, shape, dtype,
      element count and whether it is replicated across a tensor-parallel group;
    * ``mixed_execution.jsonl`` (rank 0, per update): for every microbatch the ingress
      groups (ranks, samples, mode) and the CP degrees of each layer's attention and MLP
      layouts;
    * ``buckets_rank{R}.jsonl``: the optimizer buckets (element range, members, bytes)
      and the update's reduce-scatter / all-gather payloads;
    * ``timeline_rank{R}.jsonl``: the accumulation audit's events with host nanoseconds
      (backward per microbatch, bucket reduce-scatters, the update, all-gathers);
    * ``optimizer_memory_rank{R}.jsonl``: bytes of the fp32 master shard, Adam moments,
      gradient shard, bf16 shard and the flat parameter / gradient buffers;
    * ``numerics_rank{R}.jsonl``: the outcome of the optimizer-shard and logical gates.

    Same files as the reference's runtime and accumulation audit write
    (experiments/sequence_dynamic_cp/runtime.py:197-208,315-336;
    accumulation_audit.py:31-39,158-167).
    """

    def __init__(self, output: str | Path, rank: int):
        self.root = Path(output)
        self.root.mkdir(parents=True, exist_ok=True)
        self.rank = rank
        self._inventory_done = False

    def _append(self, name: str, record: dict) -> None:
        with (self.root / name).open("a") as f:
            f.write(json.dumps(record, sort_keys=True) + "\n")

    def model_inventory(self, model) -> None:
        if self.rank != 0 or self._inventory_done:
            return
        params = [{"name": n, "shape": list(p.shape), "dtype": str(p.dtype).replace("torch.", ""),
                   "numel": p.numel(), "tp_replicated": bool(getattr(p, "tp_replicated", False))}
                  for n, p in model.named_parameters()]
        (self.root / "model_inventory.json").write_text(json.dumps(
            {"parameters": params, "total_numel": sum(p["numel"] for p in params)}, indent=1))
        self._inventory_done = True

    @staticmethod
    def _groups(layout) -> list:
        return [{"ranks": list(g.ranks), "samples": list(g.samples), "cp": len(g.ranks)} for g in layout.groups]

    def step(self, step: int, trainer, plan) -> None:
        self.model_inventory(trainer.model)
        if self.rank == 0:
            mbs = []
            for i, mb in enumerate(plan.microbatches):
                mbs.append({"microbatch": i, "ingress": self._groups(mb.ingress), "mode": mb.ingress.mode,
                            "layer_cp": [{"attention": sorted({len(g.ranks) for g in a.groups}),
                                          "mlp": sorted({len(g.ranks) for g in m.groups})} for a, m in mb.layers]})
            self._append("mixed_execution.jsonl", {"step": step, "microbatches": mbs})
        opt = trainer.optimizer
        flat = opt.flat
        self._append(f"buckets_rank{self.rank}.jsonl", {
            "step": step, "buckets": [{"index": b, "lo": lo, "hi": hi, "members": len(mem), "bytes": (hi - lo) * 4}
                                      for b, (lo, hi, mem) in enumerate(flat.buckets)],
            "reduce_scatter_bytes": opt.stats.get("reduce_scatter_bytes", 0),
            "all_gather_bytes": opt.stats.get("all_gather_bytes", 0),
            "overlapped_buckets": opt.stats.get("overlapped_buckets", 0)})
        if trainer.audit is not None:
            self._append(f"timeline_rank{self.rank}.jsonl", {"step": step, "events": trainer.audit.timeline()})

        def nbytes(t):
            return int(t.numel() * t.element_size()) if t is not None else 0
        self._append(f"optimizer_memory_rank{self.rank}.jsonl", {
            "step": step, "master": nbytes(opt.master), "exp_avg": nbytes(opt.m), "exp_avg_sq": nbytes(opt.v),
            "grad_shard": nbytes(opt.grad_shard), "param_shard_bf16": nbytes(opt.shard_bf16),
            "flat_params": nbytes(flat.flat), "flat_grads": nbytes(flat.grad)})
        gates = {}
        if trainer.numerics is not None:
            gates["optimizer"] = {"mode": trainer.numerics.mode, "failures": len(trainer.numerics.failures)}
        if trainer.logical is not None:
            gates["logical"] = {"mode": trainer.logical.mode, "failures": len(trainer.logical.failures)}
        if gates:
            self._append(f"numerics_rank{self.rank}.jsonl", {"step": step, **gates})


def step_record(step: int, loss: float, grad_norm: float, elapsed_ms: float, local_ms: float, *, tokens: int,
                loss_tokens: int, samples: int, microbatches: int, peak_allocated: int, peak_reserved: int,
                memory_budget: int, memory_required: int, admitted: bool, external_before: int = 0,
                external_after: int = 0, sync: dict | None = None, forwards: int | None = None,
                backwards: int | None = None, finite: bool = True, parameter_sync: bool = True) -> dict:
    forwards = microbatches if forwards is None else forwards
    backwards = microbatches if backwards is None else backwards
    return {"step": step, "losses": {"lm loss": loss}, "grad_norm": grad_norm, "elapsed_ms": elapsed_ms,
            "local_elapsed_ms": local_ms, "peak_allocated": peak_allocated, "peak_reserved": peak_reserved,
            "tokens": tokens, "effective_loss_tokens": loss_tokens, "samples": samples,
            "execution_microbatches_per_update": microbatches, "sync": sync or {},
            "memory_budget_bytes": memory_budget, "memory_required_bytes": memory_required,
            "external_before": external_before, "external_after": external_after,
            "all_ranks_memory_admitted": admitted, "optimizer_updates": 1, "skipped_updates": 0,
            "packet_fb": {"forwards": forwards, "backwards": backwards}, "finite": finite,
            "parameter_sync_completed": parameter_sync}


def compress(folder: str | Path, world: int) -> Path:
    """Fold ``steps_rank*.jsonl`` into ``steps_by_rank.json.gz`` (lossless)."""
    folder = Path(folder)
    data = {}
    for r in range(world):
        p = folder / f"steps_rank{r}.jsonl"
        data[str(r)] = [json.loads(x) for x in p.read_text().splitlines() if x.strip()] if p.exists() else []
    out = folder / "steps_by_rank.json.gz"
    with gzip.open(out, "wt", encoding="utf-8") as f:
        json.dump(data, f)
    return out


def _load_ranks(folder: Path, world: int):
    compact = folder / "steps_by_rank.json.gz"
    if compact.exists():
        with gzip.open(compact, "rt", encoding="utf-8") as f:
            saved = json.load(f)
        return [saved.get(str(r), []) for r in range(world)]
    ranks = []
    for r in range(world):
        p = folder / f"steps_rank{r}.jsonl"
        ranks.append([json.loads(x) for x in p.read_text().splitlines() if x.strip()] if p.exists() else [])
    return ranks


def summarize_records(folder, manifest: dict, total_steps: int, measured_steps, expected_batches: int,
                      world: int = 16) -> dict:
    folder = Path(folder)
    ranks = _load_ranks(folder, world)
    flat = [row for rows in ranks for row in rows]
    out = {"source": str(folder), "records": len(flat),
           "steps_by_rank": {r: [x["step"] for x in rows] for r, rows in enumerate(ranks)}}
    if not flat:
        return dict(out, status="no_complete_update_records")
    out["peak_bytes"] = {k: max(x[k] for x in flat) for k in ("peak_allocated", "peak_reserved",
                                                               "memory_required_bytes")}
    out["peak_GiB"] = {k: v / 2 ** 30 for k, v in out["peak_bytes"].items()}
    out["minimum_memory_budget_bytes"] = min(x["memory_budget_bytes"] for x in flat)
    checks = {
        "input_tokens": all(x["tokens"] == manifest["input_tokens"] for x in flat),
        "effective_loss_tokens": all(x["effective_loss_tokens"] == manifest["loss_tokens"] for x in flat),
        "full_update": all(x["optimizer_updates"] == 1 and x["skipped_updates"] == 0 for x in flat),
        "finite": all(x["finite"] for x in flat),
        "parameters_synchronized": all(x["parameter_sync_completed"] for x in flat),
        "forward_backward": all(x["execution_microbatches_per_update"] == expected_batches
                                and x["packet_fb"]["forwards"] == x["packet_fb"]["backwards"] == expected_batches
                                for x in flat),
        "physical_memory": all(x["all_ranks_memory_admitted"] for x in flat)}
    out["checks"] = checks
    if not all(v for k, v in checks.items() if k != "physical_memory"):
        return dict(out, status="training_contract_failed")
    if not checks["physical_memory"]:
        return dict(out, status="actual_memory_guard_rejected",
                    first_rejected_step=min(x["step"] for x in flat if not x["all_ranks_memory_admitted"]))
    if any([x["step"] for x in rows] != list(range(1, total_steps + 1)) for rows in ranks):
        return dict(out, status="incomplete")
    times = [max(rows[s - 1]["elapsed_ms"] for rows in ranks) / 1000 for s in measured_steps]
    return dict(out, status="complete", measured_steps=list(measured_steps), rankmax_seconds=times,
                mean_seconds=sum(times) / len(times))


def finite(value) -> bool:
    """Recursive finite check over nested step results (numbers, tensors, dicts, sequences)."""
    import math

    import torch
    if isinstance(value, torch.Tensor):
        return bool(torch.isfinite(value).all())
    if isinstance(value, float):
        return math.isfinite(value)
    if isinstance(value, dict):
        return all(finite(v) for v in value.values())
    if isinstance(value, (list, tuple)):
        return all(finite(v) for v in value)
    return True
