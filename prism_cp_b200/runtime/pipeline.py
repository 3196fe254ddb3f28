"""1F1B pipeline parallelism over CP stages.

The world of W ranks is cut into ``pp`` consecutive stages of W / pp ranks.
Stage s owns layers [s * L / pp, (s + 1) * L / pp) (the embedding on stage 0,
final norm, head and loss on the last stage) and runs the global batch's
plan on its own ranks: plans, layouts and CP teams are over the W / pp ranks of
one stage, and stage rank r exchanges activations and their gradients with
rank r of the neighbouring stages in the microbatch's ingress layout, so the
boundary tensors have the same rows on both sides. The schedule is 1F1B
(Narayanan et al., 2021; the reference's retired ``1f1b/`` scheduler):

    warm-up   min(pp - 1 - s, M) forwards
    steady    one forward, then one backward, M - warm-up times
    cool-down the remaining backwards

Sends and receives are NCCL point-to-point; a forward send is posted together
with the receive of the next gradient (and a gradient send with the receive of
the next activation) so neighbouring stages never wait on each other's
ordering, and the communication runs while the other stream of work proceeds.
Per step the trainer records the compute time of every microbatch on the
device, the time spent waiting for peers, and the bubble fraction
1 - compute / step (all max over ranks).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..parallel.teams import Teams
from .executor import LayoutCache, MicrobatchRun
from .optimizer import DistributedAdamW, FlatParameters
from .trainer import StepResult


@dataclass
class StageInfo:
    pp: int
    stage: int
    stage_world: int
    stage_rank: int
    first_layer: int
    num_layers: int
    group: object           # all ranks of this stage (None when the stage has one rank)
    prev: int | None        # global rank of the same stage rank on the previous stage
    next: int | None


def make_stage(pp: int, num_layers: int) -> StageInfo:
    world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
    rank = dist.get_rank() if world > 1 else 0
    if world % pp or num_layers % pp:
        raise ValueError("world size and layer count must be multiples of the pipeline size")
    ws = world // pp
    stage, srank = rank // ws, rank % ws
    groups = {}
    for s in range(pp):
        members = list(range(s * ws, (s + 1) * ws))
        groups[s] = dist.new_group(members) if (ws > 1 and world > 1) else None
    per = num_layers // pp
    return StageInfo(pp, stage, ws, srank, stage * per, per, groups[stage],
                     rank - ws if stage > 0 else None, rank + ws if stage < pp - 1 else None)


class StageTeams(Teams):
    """CP teams over the ranks of one pipeline stage (stage rank r = global rank base + r)."""

    def __init__(self, info: StageInfo):
        self.initialized = dist.is_available() and dist.is_initialized()
        self.world, self.rank = info.stage_world, info.stage_rank
        base = info.stage * info.stage_world
        self.rank_map = [base + r for r in range(self.world)]
        self.groups = {}
        self._world_group = info.group
        from ..parallel.teams import dyadic_intervals
        if self.initialized and dist.get_world_size() > 1:
            for ranks in dyadic_intervals(self.world):
                for s in range(info.pp):
                    members = [s * self.world + r for r in ranks]
                    if len(ranks) == 1:
                        group = None
                    elif len(ranks) == self.world:
                        group = None  # the stage group, created by make_stage
                    else:
                        group = dist.new_group(members)
                    if s == info.stage and self.rank in ranks:
                        self.groups[ranks] = info.group if len(ranks) == self.world else group


class PipelineTrainer:
    def __init__(self, model, info: StageInfo, device, lr=3e-4, min_lr=3e-5, weight_decay=0.1, clip_grad=1.0,
                 warmup_steps=0, decay_steps=1000, records: str | None = None, recompute_tokens: int | None = None):
        self.model, self.info, self.device = model, info, device
        # microbatches above this many tokens on a rank recompute this stage's layers in the backward
        self.recompute_tokens = recompute_tokens
        self.teams = StageTeams(info)
        self.cache = LayoutCache(info.stage_world, info.stage_rank, device, self.teams)
        self.flat = FlatParameters(model, info.stage_world)
        self.optimizer = DistributedAdamW(self.flat, group=info.group, lr=lr, min_lr=min_lr,
                                          weight_decay=weight_decay, clip_grad=clip_grad, warmup_steps=warmup_steps,
                                          decay_steps=decay_steps, world=info.stage_world)
        self.first = info.stage == 0
        self.last = info.stage == info.pp - 1
        self.stats = {}
        self.recorder = None
        if records:
            from .records import StepRecorder
            rank = dist.get_rank() if (dist.is_available() and dist.is_initialized()) else 0
            self.recorder = StepRecorder(records, rank)

    def prepare(self, batch, plan, pin: bool = True):
        from .batch import local_inputs
        return [local_inputs(batch, mb.ingress, self.info.stage_world, self.info.stage_rank,
                             pin=pin and self.device.type == "cuda") for mb in plan.microbatches]

    # ------------------------------------------------------------------ p2p
    def _exchange(self, send=None, send_to=None, recv_shape=None, recv_from=None, dtype=None):
        ops, recv = [], None
        if send is not None:
            ops.append(dist.P2POp(dist.isend, send.contiguous(), send_to))
        if recv_shape is not None:
            recv = torch.empty(recv_shape, dtype=dtype, device=self.device)
            ops.append(dist.P2POp(dist.irecv, recv, recv_from))
        if ops:
            t0 = time.perf_counter()
            for req in dist.batch_isend_irecv(ops):
                req.wait()
            self.stats["wait_s"] = self.stats.get("wait_s", 0.0) + time.perf_counter() - t0
        return recv

    # ------------------------------------------------------------------ step
    def train_step(self, batch, plan, inputs=None) -> StepResult:
        info = self.info
        if inputs is None:
            inputs = self.prepare(batch, plan)
        lengths = batch.lengths
        M = len(plan.microbatches)
        runs = [MicrobatchRun(mb, lengths, self.cache, info.first_layer, info.num_layers,
                              recompute_tokens=self.recompute_tokens)
                for mb in plan.microbatches]
        h = self.model.cfg.hidden_size
        dtype = next(self.model.parameters()).dtype
        shapes = [(run.ingress.tokens, h) for run in runs]
        self.flat.zero_grad()
        self.stats = {"wait_s": 0.0}
        loss_acc = torch.zeros((), dtype=torch.float32, device=self.device)
        saved: dict[int, tuple] = {}
        compute_events = []
        stream = torch.cuda.current_stream() if self.device.type == "cuda" else None

        def timed(fn):
            if stream is None:
                return fn()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = fn()
            b.record(stream)
            compute_events.append((a, b))
            return out

        def forward(m, x_in):
            run = runs[m]
            host = inputs[m]
            dev = host.to(self.device) if host.tokens.device != self.device else host

            def body():
                x = self.model.embed(dev.tokens) if self.first else x_in
                y, prev = run.forward_layers(self.model, x)
                from ..parallel.transport import move
                y = move(y, prev, run.ingress)
                if self.last:
                    loss, _ = self.model.loss(y, dev.labels, dev.weights)
                    return loss
                return y
            out = timed(body)
            saved[m] = (x_in, out)
            if self.last:
                loss_acc.add_(out.detach())
            return out

        def backward(m, grad):
            x_in, out = saved.pop(m)

            def body():
                if self.last:
                    out.backward()
                else:
                    torch.autograd.backward(out, grad)
            timed(body)
            return x_in.grad if (x_in is not None and not self.first) else None

        warm = min(info.pp - 1 - info.stage, M)
        t_start = time.perf_counter()
        # warm-up forwards
        for m in range(warm):
            x = None
            if not self.first:
                x = self._exchange(recv_shape=shapes[m], recv_from=info.prev, dtype=dtype).requires_grad_(True)
            y = forward(m, x)
            if not self.last:
                self._exchange(send=y.detach(), send_to=info.next)
        # steady 1F1B
        x_next = None
        if warm < M and not self.first:
            x_next = self._exchange(recv_shape=shapes[warm], recv_from=info.prev, dtype=dtype).requires_grad_(True)
        for i in range(M - warm):
            m_f, m_b = warm + i, i
            y = forward(m_f, x_next)
            g = None
            if not self.last:
                g = self._exchange(send=y.detach(), send_to=info.next, recv_shape=shapes[m_b], recv_from=info.next,
                                   dtype=dtype)
            dx = backward(m_b, g)
            last_f = m_f + 1 >= M
            if not self.first:
                x_next = self._exchange(send=dx, send_to=info.prev,
                                        recv_shape=None if last_f else shapes[m_f + 1], recv_from=info.prev,
                                        dtype=dtype)
                if x_next is not None:
                    x_next.requires_grad_(True)
        # cool-down backwards
        for m_b in range(M - warm, M):
            g = None
            if not self.last:
                g = self._exchange(recv_shape=shapes[m_b], recv_from=info.next, dtype=dtype)
            dx = backward(m_b, g)
            if not self.first:
                self._exchange(send=dx, send_to=info.prev)
        # update: gradients reduce inside the stage; the clip norm spans all stages
        opt = self.optimizer
        opt.flat.fold_param_grads()
        opt.reduce_gradients()
        sq = opt.grad_norm_sq()
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            total = sq.clone()
            dist.all_reduce(total)
            sq.copy_(total / info.stage_world)
        lr = self._apply(opt)
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        step_s = time.perf_counter() - t_start
        compute_ms = sum(a.elapsed_time(b) for a, b in compute_events) if compute_events else 0.0
        loss_t = loss_acc.clone()
        stats = torch.tensor([step_s * 1e3, compute_ms, self.stats["wait_s"] * 1e3], dtype=torch.float64,
                             device=self.device)
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(loss_t)                        # only last-stage ranks contribute
            dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        step_ms, comp_ms, wait_ms = stats.tolist()
        tokens = sum(lengths.values())
        extra = {"pipeline_stages": info.pp, "bubble_fraction": max(0.0, 1.0 - comp_ms / step_ms) if step_ms else 0.0,
                 "exposed_p2p_ms": wait_ms, "step_ms": step_ms, "compute_ms": comp_ms}
        loss = float(loss_t.item())
        if self.recorder is not None:
            from .records import step_record
            cuda = self.device.type == "cuda"
            rec = step_record(
                opt.step_count, loss, float(opt.sumsq.sqrt().item()), step_ms, step_ms, tokens=tokens,
                loss_tokens=batch.loss_tokens, samples=len(lengths), microbatches=M,
                peak_allocated=torch.cuda.max_memory_allocated(self.device) if cuda else 0,
                peak_reserved=torch.cuda.max_memory_reserved(self.device) if cuda else 0,
                memory_budget=0, memory_required=0, admitted=True, sync=dict(opt.stats),
                finite=math.isfinite(loss))
            rec["pipeline"] = dict(extra, stage=info.stage)
            self.recorder.write(rec)
        return StepResult(loss, loss_t, tokens, M, lr, elapsed_ms=step_ms, extra=extra)

    def _apply(self, opt: DistributedAdamW) -> float:
        """AdamW on the stage's shard using the already-combined squared norm."""
        import math
        from ..ops._lib import is_cuda, lib
        opt.step_count += 1
        lr = opt.current_lr(opt.step_count)
        b1, b2 = opt.betas
        bc1, bc2 = 1 - b1 ** opt.step_count, 1 - b2 ** opt.step_count
        if is_cuda(opt.master):
            if opt.weight_decay:
                opt.master.mul_(1.0 - lr * opt.weight_decay * opt.wd_mask)
            lib().adamw_step(opt.master, opt.grad_shard, opt.m, opt.v, opt.shard_bf16, opt.sumsq, opt.clip_grad,
                             lr, b1, b2, opt.eps, 0.0, bc1, bc2)
        else:
            ss = float(opt.sumsq.item())
            coef = min(1.0, opt.clip_grad / (math.sqrt(ss) + 1e-6)) if opt.clip_grad > 0 else 1.0
            if math.isfinite(ss):
                g = opt.grad_shard * coef
                opt.master.mul_(1.0 - lr * opt.weight_decay * opt.wd_mask)
                opt.m.mul_(b1).add_(g, alpha=1 - b1)
                opt.v.mul_(b2).addcmul_(g, g, value=1 - b2)
                opt.master.sub_(lr * ((opt.m / bc1) / ((opt.v / bc2).sqrt() + opt.eps)))
                opt.shard_bf16.copy_(opt.master)
        opt.gather_parameters()
        return lr
