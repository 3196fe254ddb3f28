"""Numerical contracts and the optimizer-shard / logical numerics gates.

* ``LogicalNumerics``: per-sample embedding Y, decoder Y, embedding dX and
  token loss rebuilt across ranks and layouts, compared with a reference run
  (reference: logical_numerics.py:11-208).

* ``contract(profile, architecture)``: named, frozen tolerance sets
  ``strict_v1``, ``cp_bf16_v2`` and ``cp_bf16_exploratory_v3`` for
  ``gdngqa_gpt`` / ``gqa_gpt`` (limits as the reference's
  numerical_contracts.py:9-54, so a run passes or fails the same limits in both);
  ``load_contract`` rejects any edited copy.
* ``TrainingNumerics``: writes (``mode="write"``) or checks (``mode="read"``) the
  fp32 master weights, gradients and Adam states of the first steps against a
  reference run, with relative-L2 / absolute limits from the contract and a
  MAX all-reduce of the failure flag so every rank stops together
  (reference: numerics.py:10-179).
* ``compare``: relative-L2 with an absolute floor, the metric all gates use.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import torch
import torch.distributed as dist

PROFILES = ("strict_v1", "cp_bf16_v2", "cp_bf16_exploratory_v3")
ARCHITECTURES = ("gdngqa_gpt", "gqa_gpt")


def contract(profile: str = "strict_v1", architecture: str = "gdngqa_gpt") -> dict:
    if profile not in PROFILES or architecture not in ARCHITECTURES:
        raise ValueError("Unknown numerical profile or architecture")
    if profile == "cp_bf16_exploratory_v3":
        c = contract("cp_bf16_v2", architecture)
        c.update(profile=profile, scope="exploratory performance admission; three Adam steps; provisional numerics")
        c["optimizer"]["gradients"] = {"relative": 0.15, "absolute": 1e-6}
        c["optimizer"]["weights"] = {"relative": 0.01, "absolute": 1e-6}
        c["optimizer"]["states"] = {"relative": 0.25, "absolute": 1e-6}
        c["logical"].update(decoder_Y=0.05, embedding_dX=0.10, token_loss=0.03)
        return c
    relaxed = profile == "cp_bf16_v2"
    y, dx, dw = (0.03, 0.04, 0.06) if architecture == "gdngqa_gpt" else (0.02, 0.03, 0.05)
    return {
        "profile": profile, "architecture": architecture,
        "scope": "BF16 CP/packing comparison over the first three Adam steps; no convergence claim",
        "optimizer": {
            "initial_weights": {"relative": 0.0 if relaxed else 1e-5, "absolute": 0.0 if relaxed else 1e-7},
            "gradients": {"relative": dw if relaxed else 0.005, "absolute": 1e-6},
            "weights": {"relative": 0.005 if relaxed else 1e-5, "absolute": 1e-6 if relaxed else 1e-7},
            "states": {"relative": 0.10 if relaxed else 0.005, "absolute": 1e-6},
        },
        "logical": {"tokens": 0.0, "positions": 0.0, "labels": 0.0, "loss_mask": 0.0, "embedding_Y": 0.0,
                    "decoder_Y": y if relaxed else 0.005, "embedding_dX": dx if relaxed else 0.005,
                    "token_loss": 0.01 if relaxed else 0.005},
        "finite_required": True, "exact_data_and_ownership": True}


def load_contract(path: str | Path | None = None) -> dict:
    data = json.loads(Path(path).read_text()) if path else contract()
    if data != contract(data["profile"], data["architecture"]):
        raise ValueError("Numerical contract differs from its frozen named version")
    values = [v for lim in data["optimizer"].values() for v in lim.values()] + list(data["logical"].values())
    if any(not math.isfinite(v) or v < 0 for v in values):
        raise ValueError("Numerical limits must be finite and nonnegative")
    return data


def compare(actual: torch.Tensor, expected: torch.Tensor, relative: float, absolute: float) -> dict:
    a, e = actual.double().flatten(), expected.double().flatten()
    if a.shape != e.shape:
        return {"ok": False, "reason": "shape"}
    diff = (a - e).norm().item()
    scale = e.norm().item()
    ok = diff <= relative * scale + absolute * math.sqrt(max(1, e.numel()))
    return {"ok": bool(ok and torch.isfinite(a).all()), "relative_l2": diff / scale if scale else diff,
            "max_abs": (a - e).abs().max().item() if a.numel() else 0.0}


class TrainingNumerics:
    """Optimizer-shard gate over the first ``steps`` updates (write or read mode)."""

    def __init__(self, output: str | Path, mode: str = "off", reference: str | Path | None = None,
                 steps: int = 3, limits: dict | None = None, rank: int = 0):
        if mode not in ("off", "write", "read"):
            raise ValueError("numerics mode must be off, write or read")
        self.output, self.mode, self.steps, self.rank = Path(output), mode, steps, rank
        self.reference = Path(reference) if reference else self.output
        self.limits = limits or contract()["optimizer"]
        self.failures: list[dict] = []

    def _file(self, root: Path, step: int, what: str) -> Path:
        return root / f"numerics_rank{self.rank}_step{step}_{what}.pt"

    def observe(self, step: int, optimizer) -> None:
        if self.mode == "off" or step > self.steps:
            return
        tensors = {"weights": optimizer.master, "gradients": optimizer.grad_shard,
                   "states": torch.cat([optimizer.m, optimizer.v])}
        if self.mode == "write":
            self.output.mkdir(parents=True, exist_ok=True)
            for k, t in tensors.items():
                torch.save(t.detach().cpu(), self._file(self.output, step, k))
            return
        for k, t in tensors.items():
            ref = torch.load(self._file(self.reference, step, k))
            lim = self.limits[k]
            res = compare(t.detach().cpu(), ref, lim["relative"], lim["absolute"])
            if not res["ok"]:
                self.failures.append(dict(res, step=step, field=k))
        flag = torch.tensor([1.0 if self.failures else 0.0], device=optimizer.master.device)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if flag.item() > 0:
            raise AssertionError(f"optimizer numerics gate failed at step {step}: {self.failures[:3]}")


class LogicalNumerics:
    """Logical per-sample gate: embedding Y, decoder Y, embedding dX and token loss.

    Every rank holds rows of its ingress layout; ``record`` keeps, for one
    microbatch, the local rows' (sample, position, token, label, weight) with
    the embedding output, the decoder output before the final norm, the
    gradient at the embedding output and the per-token loss. ``finish`` gathers
    all ranks' rows (``all_gather_object``), rebuilds every logical sample in
    position order, and either writes the samples (``mode="write"``, the
    reference run, typically CP = 1) or compares them with the reference: data
    fields exactly (the same token / label / mask at every position, every
    position owned once), Y / dX / loss by relative L2 under the contract's
    logical limits. The failure flag is MAX-all-reduced so all ranks stop
    together (reference: logical_numerics.py:11-208, with zigzag positions).
    """

    def __init__(self, output: str | Path, mode: str = "off", reference: str | Path | None = None, steps: int = 1,
                 limits: dict | None = None, rank: int = 0, group=None, device="cpu", distributed: bool = True):
        if mode not in ("off", "write", "read"):
            raise ValueError("logical numerics mode must be off, write or read")
        self.output, self.mode, self.steps, self.rank, self.group = Path(output), mode, steps, rank, group
        self.device = device
        # a one-process reference run inside a distributed job gathers nothing
        self.distributed = distributed
        self.reference = Path(reference) if reference else self.output
        self.limits = limits or contract("cp_bf16_v2")["logical"]
        self.rows: list[dict] = []
        self.failures: list[dict] = []

    def active(self, step: int) -> bool:
        return self.mode != "off" and step <= self.steps

    def _multi(self) -> bool:
        return (self.distributed and dist.is_available() and dist.is_initialized()
                and dist.get_world_size(self.group) > 1)

    def record(self, layout, tokens, labels, weights, y_embed, y_decoder, dx_embed, token_loss) -> None:
        """Local rows of one microbatch in ``layout`` (a LocalLayout: spans of (sample, begin, _, count))."""
        row = 0
        for sample, begin, _, count in layout.spans:
            sl = slice(row, row + count)
            self.rows.append({
                "sample": int(sample), "positions": list(range(begin, begin + count)),
                "tokens": tokens[sl].cpu(), "labels": labels[sl].cpu(), "weights": weights[sl].float().cpu(),
                "embedding_Y": y_embed[sl].float().cpu(), "decoder_Y": y_decoder[sl].float().cpu(),
                "embedding_dX": dx_embed[sl].float().cpu(), "token_loss": token_loss[sl].float().cpu()})
            row += count

    def _assemble(self, rows: list[dict]) -> dict:
        by_sample: dict = {}
        for r in rows:
            by_sample.setdefault(r["sample"], []).append(r)
        out = {}
        for s, parts in by_sample.items():
            n = max(p for r in parts for p in r["positions"]) + 1
            owned = torch.zeros(n, dtype=torch.int32)
            fields = {}
            for r in parts:
                idx = torch.tensor(r["positions"])
                owned[idx] += 1
                for k in ("tokens", "labels", "weights", "embedding_Y", "decoder_Y", "embedding_dX", "token_loss"):
                    t = r[k]
                    if k not in fields:
                        fields[k] = torch.zeros((n,) + tuple(t.shape[1:]), dtype=t.dtype)
                    fields[k][idx] = t
            fields["owned"] = owned
            out[s] = fields
        return out

    def finish(self, step: int) -> None:
        if not self.active(step):
            self.rows = []
            return
        rows = self.rows
        self.rows = []
        if self._multi():
            gathered = [None] * dist.get_world_size(self.group)
            dist.all_gather_object(gathered, rows, group=self.group)
            rows = [r for part in gathered for r in part]
        samples = self._assemble(rows)
        failures = []
        if self.rank == 0:
            if self.mode == "write":
                self.output.mkdir(parents=True, exist_ok=True)
                torch.save(samples, self.output / f"logical_step{step}.pt")
            else:
                ref = torch.load(self.reference / f"logical_step{step}.pt")
                if set(ref) != set(samples):
                    failures.append({"step": step, "field": "samples", "reason": "sample sets differ"})
                for s in set(ref) & set(samples):
                    a, e = samples[s], ref[s]
                    if not torch.equal(a["owned"], torch.ones_like(a["owned"])):
                        failures.append({"step": step, "sample": s, "field": "ownership"})
                    for k in ("tokens", "labels", "weights"):
                        if not torch.equal(a[k], e[k]):
                            failures.append({"step": step, "sample": s, "field": k})
                    for k in ("embedding_Y", "decoder_Y", "embedding_dX", "token_loss"):
                        res = compare(a[k], e[k], self.limits[k], 0.0)
                        if not res["ok"]:
                            failures.append(dict(res, step=step, sample=s, field=k))
        self.failures.extend(failures)
        flag = torch.tensor([1.0 if failures else 0.0], device=self.device)
        if self._multi():
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        if flag.item() > 0:
            raise AssertionError(f"logical numerics gate failed at step {step}: {failures[:3]}")
