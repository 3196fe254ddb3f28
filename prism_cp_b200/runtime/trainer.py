"""Training step over a plan: microbatch loop, gradient sync, AdamW, guards.

``Trainer.train_step(batch, plan)`` is the public entry point: it copies each
microbatch's inputs from (pinned) host memory, runs forward/backward through
the plan-driven executor, accumulates fp32 gradients, reduce-scatters them,
clips, applies the distributed AdamW and all-gathers the parameters, then
returns a ``StepResult``. Guards follow the reference's contract
(experiments/sequence_dynamic_cp/runtime.py:392-518): finite loss/grad check,
HBM admission ``peak + external <= min(0.9 total, total - 8 GiB)`` agreed across
ranks with an all-reduce MIN, and rank-max step time.
"""

from __future__ import annotations

import math
import os
import sys
import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..planner.joint.ir import Plan
from .audits import AccumulationAudit, PacketAccounting, TokenwiseFusionAudit
from .batch import GlobalBatch, HostInputs, local_inputs
from .executor import LayoutCache, MicrobatchRun
from .optimizer import DistributedAdamW, FlatParameters
from .records import RunRecords, StepRecorder, step_record
from ..utils import watchdog
from ..utils.tracing import nvtx


DEBUG_SYNC = os.environ.get("PRISM_DEBUG_SYNC", "0") in ("1", "2")
# transport of the CP-transition reshard on CUDA: "p2p" (gather over NVLink, default) or "nccl" (all-to-all)
RESHARD = os.environ.get("PRISM_RESHARD", "p2p")


def hbm_budget(total_bytes: int) -> int:
    return min(int(0.9 * total_bytes), total_bytes - 8 * 1024 ** 3)


@dataclass
class StepResult:
    loss: float
    loss_tensor: torch.Tensor
    tokens: int
    microbatches: int
    lr: float
    elapsed_ms: float | None = None
    grad_norm: float | None = None
    peak_allocated: int | None = None
    admitted: bool = True
    extra: dict = field(default_factory=dict)


class Trainer:
    def __init__(self, model, teams, device, lr=3e-4, min_lr=3e-5, weight_decay=0.1, clip_grad=1.0,
                 warmup_steps=0, decay_steps=1000, group=None, hbm_guard=True, records: str | None = None,
                 numerics=None, audit: bool = False, overlap_grad_reduce: bool = False,
                 bucket_bytes: int = 256 << 20, logical=None, recompute_tokens: int | None = None,
                 overlap_param_gather: bool = False):
        self.model, self.teams, self.device = model, teams, device
        self.world = teams.world
        self.rank = teams.rank
        tp = getattr(model, "tp", None)
        self.tp = tp if (tp is not None and tp.enabled) else None
        if group is None and self.tp is not None:
            # every TP index updates its own copy of the model; shards never mix across indices
            group = teams.world_group
        self.group = group
        bucketed = overlap_grad_reduce or overlap_param_gather
        self.flat = FlatParameters(model, self.world, bucket_bytes=bucket_bytes if bucketed else None)
        self.optimizer = DistributedAdamW(self.flat, group=group, lr=lr, min_lr=min_lr,
                                          weight_decay=weight_decay, clip_grad=clip_grad,
                                          warmup_steps=warmup_steps, decay_steps=decay_steps, world=self.world,
                                          tp_group=self.tp.group if self.tp is not None else None)
        self.overlap = self.optimizer.enable_overlap() if overlap_grad_reduce else None
        if device.type == "cuda" and self.world > 1 and self.tp is None and RESHARD == "p2p":
            # CP-transition reshards pull their rows over NVLink from a symmetric heap (one gather
            # kernel per reshard) instead of an NCCL all-to-all
            from ..parallel import transport
            from ..parallel.symm import P2PTransport
            transport.use_p2p(P2PTransport(group=teams.world_group, device=device))
        self.param_gather = self.optimizer.enable_param_gather_overlap(model) if overlap_param_gather else None
        self.cache = LayoutCache(self.world, self.rank, device, teams)
        self.hbm_guard = hbm_guard and device.type == "cuda"
        self.loss_acc = torch.zeros((), dtype=torch.float32, device=device)
        # record files are per process: under TP several ranks share one logical rank
        rec_rank = dist.get_rank() if (dist.is_available() and dist.is_initialized()) else self.rank
        self.recorder = StepRecorder(records, rec_rank) if records else None
        self.run_records = RunRecords(records, rec_rank) if records else None
        self.numerics = numerics
        self.logical = logical
        if logical is not None and logical.group is None and self.group is not None:
            # rebuild logical samples from the ranks of this TP index only (the others hold copies)
            logical.group = self.group
        self.audit = AccumulationAudit() if audit else None
        # audited steps also check tokenwise fusion and per-microbatch F/B accounting
        self.fusion = TokenwiseFusionAudit(model) if audit else None
        self.packets = PacketAccounting(memory_samples=audit and device.type == "cuda") if audit else None
        self.step_index = 0
        self.watchdog = watchdog.from_env()
        # microbatches above this many tokens on a rank recompute their layers in the backward
        self.recompute_tokens = recompute_tokens

    # ------------------------------------------------------------------ inputs
    def prepare(self, batch: GlobalBatch, plan: Plan, pin: bool = True) -> list[HostInputs]:
        return [local_inputs(batch, mb.ingress, self.world, self.rank, pin=pin and self.device.type == "cuda")
                for mb in plan.microbatches]

    # ------------------------------------------------------------------ step
    def forward_backward(self, batch_lengths: dict, plan: Plan, inputs: list):
        # embedding, final norm and head; the layers wait for their own gathers in pre-hooks
        self.optimizer.wait_parameters(top_only=True)
        self.loss_acc.zero_()
        last = len(plan.microbatches) - 1
        for index, (mb, host) in enumerate(zip(plan.microbatches, inputs)):
            dev = host.to(self.device) if host.tokens.device != self.device else host
            run = MicrobatchRun(mb, batch_lengths, self.cache, recompute_tokens=self.recompute_tokens)
            watchdog.beat(f"step {self.step_index + 1} microbatch {index} forward")
            logical = self.logical is not None and self.logical.active(self.step_index + 1)
            with nvtx(f"microbatch {index} forward"):
                if logical:
                    from ..parallel.transport import move
                    x0 = self.model.embed(dev.tokens)
                    x0.retain_grad()
                    y, prev = run.forward_layers(self.model, x0)
                    y = move(y, prev, run.ingress)
                    loss, ce = self.model.loss(y, dev.labels, dev.weights)
                else:
                    loss, _ = run.forward(self.model, dev.tokens, dev.labels, dev.weights, self.packets,
                                          self.optimizer.step_count)
            self._debug_point(index, "forward")
            if self.overlap is not None:
                # the last backward reduce-scatters each finished bucket while it runs
                self.overlap.arm(index == last)
            watchdog.beat(f"step {self.step_index + 1} microbatch {index} backward")
            with nvtx(f"microbatch {index} backward"):
                loss.backward()
            if logical:
                self.logical.record(run.ingress, dev.tokens, dev.labels, dev.weights, x0.detach(), y.detach(),
                                    x0.grad, ce)
            self._debug_point(index, "backward")
            if self.audit is not None:
                self.audit.backward(len(self.audit.events))
            self.loss_acc += loss.detach()
        if self.world > 1:
            dist.all_reduce(self.loss_acc, op=dist.ReduceOp.SUM, group=self.group)
        return self.loss_acc

    def _debug_point(self, index: int, phase: str) -> None:
        """With PRISM_DEBUG_SYNC=1: synchronise, check the kernels' status word and log progress."""
        if not DEBUG_SYNC or self.device.type != "cuda":
            return
        t0 = time.perf_counter()
        torch.cuda.synchronize(self.device)
        from ..ops._lib import check_status
        check_status(self.device)
        print(f"[debug] step {self.step_index} microbatch {index} {phase} done, waited "
              f"{time.perf_counter() - t0:.3f}s, allocated {torch.cuda.memory_allocated(self.device) / 2**30:.1f} GiB, "
              f"reserved {torch.cuda.memory_reserved(self.device) / 2**30:.1f} GiB", file=sys.stderr, flush=True)

    def train_step(self, batch: GlobalBatch, plan: Plan, inputs: list | None = None,
                   read_loss: bool = True) -> StepResult:
        if inputs is None:
            inputs = self.prepare(batch, plan)
        track = self.recorder is not None or self.audit is not None
        if track:
            return self._tracked_step(batch, plan, inputs)
        self.flat.zero_grad()
        loss = self.forward_backward(batch.lengths, plan, inputs)
        if self.logical is not None:
            self.logical.finish(self.step_index + 1)
        watchdog.beat(f"step {self.step_index + 1} optimizer")
        lr = self.optimizer.step()
        self.step_index += 1
        watchdog.beat(f"step {self.step_index} done")
        value = float(loss.item()) if read_loss else float("nan")
        if read_loss and not math.isfinite(value):
            raise FloatingPointError("non-finite loss in training step")
        return StepResult(value, loss, batch.total_tokens, len(plan.microbatches), lr)

    def _tracked_step(self, batch: GlobalBatch, plan: Plan, inputs: list) -> StepResult:
        """A step with records, audit and guards (reference: runtime.py:392-518)."""
        cuda = self.device.type == "cuda"
        if cuda:
            torch.cuda.synchronize(self.device)
            torch.cuda.reset_peak_memory_stats(self.device)
        if self.world > 1:
            dist.barrier()
        external_before = self._external() if cuda else 0
        t0 = time.perf_counter()
        if self.audit is not None:
            self.audit.events.clear()
            self.audit.times.clear()
            self.fusion.reset()
            self.packets.begin(self.optimizer.step_count, len(plan.microbatches))
        self.flat.zero_grad()
        loss = self.forward_backward(batch.lengths, plan, inputs)
        if self.logical is not None:
            self.logical.finish(self.step_index + 1)
        if self.audit is not None:
            logical = self.logical is not None and self.logical.active(self.step_index + 1)
            self.fusion.check(len(plan.microbatches))
            if not logical:
                self.last_packet = self.packets.finish(self.optimizer.step_count)
            self.optimizer.audit = self.audit
        lr = self.optimizer.step()
        self.step_index += 1
        if cuda:
            torch.cuda.synchronize(self.device)
        local_ms = (time.perf_counter() - t0) * 1000
        elapsed = torch.tensor([local_ms], dtype=torch.float64, device=self.device)
        if self.world > 1:
            dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        value = float(loss.item())
        grad_norm = float(self.optimizer.sumsq.sqrt().item())
        finite_ok = math.isfinite(value) and math.isfinite(grad_norm)
        admitted, mem = self.admission()
        self.optimizer.wait_parameters()
        if self.numerics is not None:
            self.numerics.observe(self.step_index, self.optimizer)
        if self.audit is not None:
            self.audit.check(len(plan.microbatches))
        if self.recorder is not None:
            self.recorder.write(step_record(
                self.step_index, value, grad_norm, float(elapsed.item()), local_ms, tokens=batch.total_tokens,
                loss_tokens=batch.loss_tokens, samples=len(batch.lengths), microbatches=len(plan.microbatches),
                peak_allocated=mem.get("peak_allocated", 0),
                peak_reserved=torch.cuda.max_memory_reserved(self.device) if cuda else 0,
                memory_budget=mem.get("budget", 0), memory_required=mem.get("required", 0), admitted=admitted,
                external_before=external_before, external_after=mem.get("external", 0),
                sync=dict(self.optimizer.stats), finite=finite_ok,
                **self._packet_counts()))
        if self.run_records is not None:
            self.run_records.step(self.step_index, self, plan)
        if not finite_ok:
            raise FloatingPointError("non-finite loss or gradient norm in training step")
        if not admitted:
            raise RuntimeError(f"HBM admission rejected the step: {mem}")
        return StepResult(value, loss, batch.total_tokens, len(plan.microbatches), lr,
                          elapsed_ms=float(elapsed.item()), grad_norm=grad_norm,
                          peak_allocated=mem.get("peak_allocated"), admitted=admitted, extra=mem)

    def _packet_counts(self) -> dict:
        """Observed forward/backward counts of the last audited step (the planned count otherwise)."""
        packet = getattr(self, "last_packet", None)
        return {} if packet is None else {"forwards": packet["forwards"], "backwards": packet["backwards"]}

    def _external(self) -> int:
        free, total = torch.cuda.mem_get_info(self.device)
        return max(0, total - free - torch.cuda.memory_reserved(self.device))

    # ------------------------------------------------------------------ guards
    def admission(self) -> tuple[bool, dict]:
        if not self.hbm_guard:
            return True, {}
        free, total = torch.cuda.mem_get_info(self.device)
        peak = torch.cuda.max_memory_allocated(self.device)
        reserved = torch.cuda.memory_reserved(self.device)
        external = max(0, total - free - reserved)
        required = peak + external
        budget = hbm_budget(total)
        ok = torch.tensor([1 if required <= budget else 0], dtype=torch.int32, device=self.device)
        if self.world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        return bool(ok.item()), dict(peak_allocated=peak, external=external, required=required, budget=budget)
