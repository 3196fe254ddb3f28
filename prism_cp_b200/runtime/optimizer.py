"""Distributed AdamW over flat buffers (Megatron ``--use-distributed-optimizer``).

All model parameters become views into one flat bf16 buffer and every
parameter gets a ``main_grad`` view into one flat fp32 gradient buffer (the
linear layers accumulate their weight gradients straight into it from the
GEMM epilogue). The flat buffers are padded to a multiple of the world size;
rank r owns shard r: fp32 master weights, Adam m and v. One update is

    reduce-scatter(grad, SUM) -> shard grad          (NCCL; gloo on CPU)
    sumsq(shard grad) -> all-reduce(SUM)             (device scalar, no host sync)
    AdamW(shard) with clip coef = min(1, max_norm / ||g||)   (one kernel)
    all-gather(bf16 shard) -> flat bf16 params

Gradient buckets (``bucket_bytes``) let the reduce-scatter of finished layers
overlap the rest of the backward on a side stream (``--overlap-grad-reduce``),
and the all-gather of the updated parameters overlap the next forward
(``--overlap-param-gather``): each bucket is gathered on a side stream and the
compute stream waits for it only when the first module that reads it runs.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops._lib import is_cuda, lib


class FlatParameters:
    """All trainable parameters as views into one flat buffer, grouped in gradient buckets.

    Without ``bucket_bytes`` there is one bucket in module order. With it, the
    parameters are laid out in backward order (last layers first) and cut into
    buckets of at least ``bucket_bytes`` of fp32 gradient, each padded to a
    multiple of 128 * world elements, so every bucket can be reduce-scattered on
    its own as soon as the backward has produced all of its gradients.
    """

    def __init__(self, model: torch.nn.Module, world: int, dtype=None, bucket_bytes: int | None = None):
        params = [p for p in model.parameters() if p.requires_grad]
        self.params = params
        device = params[0].device
        # the flat buffer keeps the model's compute dtype (bf16 on GPU, fp32 for CPU oracles)
        if dtype is None:
            dtype = torch.bfloat16 if any(p.dtype == torch.bfloat16 for p in params) else params[0].dtype
        # every parameter starts on a 128-byte boundary (TMA and vector kernels need
        # 16-byte aligned operands); the gaps are zero and never updated
        def slot(n):
            return (n + 63) // 64 * 64

        def pad(n):
            return (n + align - 1) // align * align

        align = 128 * world
        order = list(range(len(params)))[::-1] if bucket_bytes else list(range(len(params)))
        starts = [0] * len(params)
        buckets, members, lo, off = [], [], 0, 0
        for i in order:
            starts[i] = off
            off += slot(params[i].numel())
            members.append(i)
            if bucket_bytes and (off - lo) * 4 >= bucket_bytes:
                off = pad(off)
                buckets.append((lo, off, tuple(members)))
                lo, members = off, []
        if members or not buckets:
            off = pad(off)
            buckets.append((lo, off, tuple(members)))
        self.buckets = buckets
        self.padded = off
        self.numel = off
        self.flat = torch.zeros(self.padded, dtype=dtype, device=device)
        self.grad = torch.zeros(self.padded, dtype=torch.float32, device=device)
        self.offsets = []
        for i, p in enumerate(params):
            o, n = starts[i], p.numel()
            view = self.flat[o:o + n].view_as(p)
            view.copy_(p.detach().to(dtype))
            p.data = view
            p.main_grad = self.grad[o:o + n].view_as(p)
            self.offsets.append((o, n))
        self.bucket_of = {}
        for b, (_, _, mem) in enumerate(buckets):
            for i in mem:
                self.bucket_of[id(params[i])] = b
        # decoupled weight decay only on matrices (Megatron excludes norms/biases/1-D)
        self.decay_mask = torch.zeros(self.padded, dtype=torch.bool, device=device)
        for p, (o, n) in zip(params, self.offsets):
            if p.dim() >= 2:
                self.decay_mask[o:o + n] = True

    def zero_grad(self):
        self.grad.zero_()
        for p in self.params:
            p.grad = None

    def fold_param_grads(self):
        """Accumulate autograd ``.grad`` of params whose ops do not write main_grad."""
        for p in self.params:
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(torch.float32))
                p.grad = None


class DistributedAdamW:
    def __init__(self, flat: FlatParameters, group=None, lr=3e-4, min_lr=3e-5, betas=(0.9, 0.95), eps=1e-8,
                 weight_decay=0.1, clip_grad=1.0, warmup_steps=0, decay_steps=1000, decay_style="cosine",
                 world: int | None = None, tp_group=None):
        self.flat = flat
        self.group = group
        self.tp_group = tp_group
        if world is None:
            world = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
        self.world = world
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        # rank r owns slice r of every bucket; the optimizer state is their concatenation
        self.slices = []
        sh = 0
        for lo, hi, _ in flat.buckets:
            size = (hi - lo) // self.world
            self.slices.append((lo, hi, lo + self.rank * size, size, sh))
            sh += size
        self.shard_size = sh
        owned = [flat.flat[a:a + n] for _, _, a, n, _ in self.slices]
        self.master = torch.cat(owned).to(torch.float32)
        self.shard_bf16 = torch.cat(owned).clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.grad_shard = torch.zeros_like(self.master)
        self.wd_mask = torch.cat([flat.decay_mask[a:a + n] for _, _, a, n, _ in self.slices]).to(torch.float32)
        # elements of tensor-parallel shards: their squared norms add up across the TP group
        self.tp_mask = None
        if tp_group is not None:
            shard = torch.zeros(flat.padded, dtype=torch.bool, device=flat.flat.device)
            for p, (o, n) in zip(flat.params, flat.offsets):
                if not getattr(p, "tp_replicated", False):
                    shard[o:o + n] = True
            self.tp_mask = torch.cat([shard[a:a + n] for _, _, a, n, _ in self.slices]).to(torch.float32)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=self.master.device)
        self.lr, self.min_lr, self.betas, self.eps = lr, min_lr, betas, eps
        self.weight_decay, self.clip_grad = weight_decay, clip_grad
        self.warmup_steps, self.decay_steps, self.decay_style = warmup_steps, decay_steps, decay_style
        self.step_count = 0
        self.stats = {"reduce_scatter_bytes": 0, "all_gather_bytes": 0, "overlapped_buckets": 0}
        self.audit = None
        self._overlap = None
        self._param_gather = None

    @property
    def lo(self) -> int:
        return self.slices[0][2]

    @property
    def hi(self) -> int:
        return self.slices[-1][2] + self.slices[-1][3]

    # -------------------------------------------------------------- schedule
    def current_lr(self, step: int) -> float:
        if self.warmup_steps and step <= self.warmup_steps:
            return self.lr * step / self.warmup_steps
        if self.decay_style == "constant":
            return self.lr
        t = min(1.0, max(0.0, (step - self.warmup_steps) / max(1, self.decay_steps)))
        if self.decay_style == "linear":
            return self.min_lr + (self.lr - self.min_lr) * (1 - t)
        return self.min_lr + 0.5 * (self.lr - self.min_lr) * (1 + math.cos(math.pi * t))

    # -------------------------------------------------------------- collectives
    def _reduce_bucket(self, b: int):
        lo, hi, _, size, sh = self.slices[b]
        g = self.flat.grad[lo:hi]
        if self.world > 1:
            dist.reduce_scatter_tensor(self.grad_shard[sh:sh + size], g, op=dist.ReduceOp.SUM, group=self.group)
            self.stats["reduce_scatter_bytes"] += g.numel() * 4
        else:
            self.grad_shard[sh:sh + size].copy_(g)
        if self.audit is not None:
            self.audit.reduce_scatter(g.numel() * 4)

    def reduce_gradients(self):
        ov = self._overlap
        done = ov.finish() if ov is not None else set()
        for b in range(len(self.slices)):
            if b not in done:
                self._reduce_bucket(b)

    def _gather_bucket(self, b: int):
        lo, hi, _, size, sh = self.slices[b]
        if self.world > 1:
            dist.all_gather_into_tensor(self.flat.flat[lo:hi], self.shard_bf16[sh:sh + size], group=self.group)
            self.stats["all_gather_bytes"] += (hi - lo) * self.flat.flat.element_size()
        else:
            self.flat.flat[lo:hi].copy_(self.shard_bf16[sh:sh + size])
        if self.audit is not None:
            self.audit.all_gather((hi - lo) * self.flat.flat.element_size())

    def gather_parameters(self):
        if self._param_gather is not None:
            self._param_gather.launch()
            return
        for b in range(len(self.slices)):
            self._gather_bucket(b)

    def wait_parameters(self, top_only: bool = False):
        """Make the current stream wait for the parameter all-gathers still in flight (only those of
        the model's own parameters with ``top_only``; the layers wait in their pre-hooks)."""
        if self._param_gather is not None:
            if top_only:
                self._param_gather.wait_top()
            else:
                self._param_gather.wait_all()

    # -------------------------------------------------------------- overlap
    def enable_overlap(self):
        """Reduce-scatter each gradient bucket on a side stream as soon as the backward
        of the last microbatch has produced all of its gradients."""
        self._overlap = _GradOverlap(self)
        return self._overlap

    def enable_param_gather_overlap(self, model: torch.nn.Module):
        """Gather each bucket's updated parameters on a side stream after the update; the compute
        stream waits per bucket in a forward pre-hook of every module that owns parameters, and for
        the model's own parameters (embedding, final norm, head) before the next forward."""
        self._param_gather = _ParamGather(self, model)
        return self._param_gather

    # -------------------------------------------------------------- update
    def grad_norm_sq(self) -> torch.Tensor:
        self.sumsq.zero_()
        if self.tp_mask is not None:
            sq = self.grad_shard.float().pow(2)
            parts = torch.stack([(sq * self.tp_mask).sum(), (sq * (1 - self.tp_mask)).sum()])
            if self.world > 1:
                dist.all_reduce(parts, op=dist.ReduceOp.SUM, group=self.group)
            shard_part = parts[:1].clone()
            dist.all_reduce(shard_part, op=dist.ReduceOp.SUM, group=self.tp_group)
            self.sumsq.copy_(shard_part + parts[1:])
            return self.sumsq
        if is_cuda(self.grad_shard):
            lib().sumsq_accumulate(self.grad_shard, self.sumsq)
        else:
            self.sumsq += self.grad_shard.pow(2).sum()
        if self.world > 1:
            dist.all_reduce(self.sumsq, op=dist.ReduceOp.SUM, group=self.group)
        return self.sumsq

    def step(self):
        # the previous gathers read shard_bf16, which this update rewrites
        self.wait_parameters()
        self.flat.fold_param_grads()
        self.reduce_gradients()
        self.grad_norm_sq()
        self.step_count += 1
        if self.audit is not None:
            self.audit.optimizer_step()
        lr = self.current_lr(self.step_count)
        b1, b2 = self.betas
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        shard_bf16 = self.shard_bf16
        if is_cuda(self.master):
            # decoupled weight decay on matrices first (p *= 1 - lr*wd), then one fused
            # AdamW launch that also writes the bf16 shard; a non-finite norm skips it
            if self.weight_decay:
                self.master.mul_(1.0 - lr * self.weight_decay * self.wd_mask)
            lib().adamw_step(self.master, self.grad_shard, self.m, self.v, shard_bf16, self.sumsq, self.clip_grad,
                             lr, b1, b2, self.eps, 0.0, bc1, bc2)
        else:
            ss = float(self.sumsq.item())
            coef = min(1.0, self.clip_grad / (math.sqrt(ss) + 1e-6)) if self.clip_grad > 0 else 1.0
            if math.isfinite(ss):
                g = self.grad_shard * coef
                self.master.mul_(1.0 - lr * self.weight_decay * self.wd_mask)
                self.m.mul_(b1).add_(g, alpha=1 - b1)
                self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
                self.master.sub_(lr * ((self.m / bc1) / ((self.v / bc2).sqrt() + self.eps)))
                shard_bf16.copy_(self.master)
        self.gather_parameters()
        return lr

    def state_dict(self):
        return {"master": self.master, "m": self.m, "v": self.v, "step": self.step_count,
                "rank": self.rank, "world": self.world, "lo": self.lo, "hi": self.hi}

    def load_state_dict(self, state):
        if state["world"] != self.world or state["lo"] != self.lo:
            raise ValueError("optimizer shard layout differs from the checkpoint")
        self.master.copy_(state["master"])
        self.m.copy_(state["m"])
        self.v.copy_(state["v"])
        self.step_count = int(state["step"])
        self.shard_bf16.copy_(self.master)
        self.gather_parameters()


class _GradOverlap:
    """Tracks which parameters of each bucket received their last gradient.

    Kernels that accumulate straight into ``main_grad`` report through
    ``ops._lib.on_main_grad``; every other parameter reports from a
    post-accumulate-grad hook, which also folds its ``.grad`` into ``main_grad``.
    While ``armed`` (the last microbatch's backward), a bucket whose parameters
    have all reported is reduce-scattered on a side stream after an event on the
    compute stream; ``finish`` makes the compute stream wait for those reduces.
    """

    def __init__(self, opt: DistributedAdamW):
        from ..ops._lib import set_grad_listener
        self.opt = opt
        flat = opt.flat
        self.need = [set(id(flat.params[i]) for i in mem) for _, _, mem in flat.buckets]
        self.seen = [set() for _ in flat.buckets]
        self.launched: set = set()
        self.armed = False
        dev = flat.grad.device
        self.side = torch.cuda.Stream(device=dev) if flat.grad.is_cuda else None
        self.handles = [p.register_post_accumulate_grad_hook(self._on_accumulated) for p in flat.params]
        set_grad_listener(self._on_main_grad)

    def arm(self, armed: bool = True):
        self.armed = armed
        if armed:
            self.seen = [set() for _ in self.seen]
            self.launched = set()

    def _on_accumulated(self, p):
        if p.grad is not None:
            p.main_grad.add_(p.grad.to(torch.float32))
            p.grad = None
        self._on_main_grad(p)

    def _on_main_grad(self, p):
        if not self.armed:
            return
        b = self.opt.flat.bucket_of.get(id(p))
        if b is None or b in self.launched:
            return
        self.seen[b].add(id(p))
        if self.seen[b] >= self.need[b]:
            self.launched.add(b)
            if self.side is None:
                self.opt._reduce_bucket(b)
                return
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self.side):
                self.side.wait_event(ev)
                self.opt._reduce_bucket(b)
            self.opt.stats["overlapped_buckets"] += 1

    def finish(self) -> set:
        done = set(self.launched)
        if self.side is not None and done:
            torch.cuda.current_stream().wait_stream(self.side)
        self.armed = False
        return done

    def close(self):
        from ..ops._lib import set_grad_listener
        for h in self.handles:
            h.remove()
        set_grad_listener(None)


class _ParamGather:
    """Parameter all-gather overlapped with the next forward (``--overlap-param-gather``).

    ``launch`` runs after the update: the side stream waits for it, then gathers first the
    buckets holding the model's own parameters (read before the first layer and by the head),
    then the layers' buckets in forward order (the flat layout is backward order, so the last
    bucket first), recording one event per bucket. A forward pre-hook on every submodule that
    owns parameters makes the compute stream wait for its buckets' events; the trainer calls
    ``wait_top`` before the first microbatch. Without a side stream (CPU) the gather is
    synchronous.
    """

    def __init__(self, opt: DistributedAdamW, model: torch.nn.Module):
        self.opt = opt
        flat = opt.flat
        self.side = torch.cuda.Stream(device=flat.flat.device) if flat.flat.is_cuda else None
        self.pending: dict = {}
        of = flat.bucket_of
        self.top = tuple(sorted({of[id(p)] for p in model.parameters(recurse=False) if id(p) in of}))
        rest = [b for b in reversed(range(len(opt.slices))) if b not in self.top]
        self.order = list(self.top) + rest
        self.handles = []
        for mod in model.modules():
            if mod is model:
                continue
            own = tuple(sorted({of[id(p)] for p in mod.parameters(recurse=False) if id(p) in of}))
            if own:
                self.handles.append(mod.register_forward_pre_hook(lambda m, args, own=own: self.wait(own)))

    def launch(self):
        if self.side is None:
            for b in self.order:
                self.opt._gather_bucket(b)
            return
        ready = torch.cuda.Event()
        ready.record()
        with torch.cuda.stream(self.side):
            self.side.wait_event(ready)
            for b in self.order:
                self.opt._gather_bucket(b)
                ev = torch.cuda.Event()
                ev.record(self.side)
                self.pending[b] = ev

    def wait(self, buckets):
        for b in buckets:
            ev = self.pending.pop(b, None)
            if ev is not None:
                torch.cuda.current_stream().wait_event(ev)

    def wait_top(self):
        self.wait(self.top)

    def wait_all(self):
        self.wait(list(self.pending))

    def close(self):
        self.wait_all()
        for h in self.handles:
            h.remove()
