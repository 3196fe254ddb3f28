"""Tensor parallelism (Megatron-style column/row parallel linears) on top of CP.

The global world of W ranks is split into W / tp logical ranks of ``tp``
consecutive GPUs each (one NVSwitch hop apart on a B200 box). Plans, layouts
and CP teams are defined over logical ranks: every tensor-parallel index
runs the same CP schedule on its own shard of the heads, with its own set of
dyadic teams (``Teams(..., rank_map=...)``), and the CP-transition reshard runs
among the ranks of one index. The residual stream is replicated inside a TP
group; attention/GDN heads and the MLP's hidden units are split:

* ``column_linear(x, w_shard)``: replicated input, output sharded by columns;
  its input gradient is summed over the group (all-reduce in the backward);
* ``row_linear(x_shard, w_shard)``: sharded input, partial outputs summed over
  the group (all-reduce in the forward, identity backward).

The sums run as reduce-scatter + all-gather (``dist``; NCCL over NVLink on
CUDA). With ``PRISM_TP_FUSED=1`` they are fused into the GEMM that produces them
instead (``tp_fused.FusedAllReduceGemm``: the tcgen05 kernel exchanges partial
and finished tiles over NVLink peer memory while it computes); that form is
correct but measured slower, see ``tp_fused``. Parameters owned by a shard reduce their gradients only over the
ranks of the same TP index; replicated parameters (norms, embedding, head,
per-value-dim norm weights) reduce over the whole world.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops._lib import aligned_rows
from ..ops.gemm import linear, matmul, weight_grad
from . import tp_fused


@dataclass
class TPContext:
    tp: int
    index: int             # this rank's position inside its TP group
    logical_rank: int
    logical_world: int
    group: object          # the TP group (None when tp == 1)
    index_group: object    # all ranks with this TP index (None when there is one logical rank)

    @property
    def enabled(self) -> bool:
        return self.tp > 1

    def rank_map(self, index: int | None = None) -> list[int]:
        """Global rank of every logical rank for one TP index."""
        i = self.index if index is None else index
        return [l * self.tp + i for l in range(self.logical_world)]


def make_tp(tp: int) -> TPContext:
    """Create the TP groups (every rank takes part in every ``new_group``)."""
    if tp <= 1 or not (dist.is_available() and dist.is_initialized()):
        world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
        rank = dist.get_rank() if world > 1 else 0
        return TPContext(1, 0, rank, world, None, dist.group.WORLD if world > 1 else None)
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % tp:
        raise ValueError("world size must be a multiple of the tensor-parallel size")
    logical_world = world // tp
    groups, index_groups = {}, {}
    for l in range(logical_world):
        groups[l] = dist.new_group([l * tp + i for i in range(tp)])
    for i in range(tp):
        index_groups[i] = dist.new_group([l * tp + i for l in range(logical_world)]) if logical_world > 1 else None
    return TPContext(tp, rank % tp, rank // tp, logical_world, groups[rank // tp], index_groups[rank % tp])


def _sum_over_group(x: torch.Tensor, group) -> torch.Tensor:
    if group is None:
        return x
    x = x.contiguous()
    n = dist.get_world_size(group)
    rows = x.shape[0]
    if x.is_cuda and rows % n == 0:
        # reduce-scatter + all-gather: the pair a fused GEMM epilogue / prologue replaces
        part = torch.empty((rows // n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(part, x, group=group)
        out = torch.empty_like(x)
        dist.all_gather_into_tensor(out, part, group=group)
        return out
    out = x.clone()
    dist.all_reduce(out, group=group)
    return out


class _CopyToTP(torch.autograd.Function):
    """Identity forward, gradient summed over the TP group (input of a column-parallel linear)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        return _sum_over_group(g, ctx.group), None


class _ReduceFromTP(torch.autograd.Function):
    """Partial outputs summed over the TP group, identity backward (row-parallel output)."""

    @staticmethod
    def forward(ctx, x, group):
        return _sum_over_group(x, group)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _ColumnLinearFused(torch.autograd.Function):
    """y = x W_shard^T with replicated x; dx = sum over the group of dy_shard W_shard (fused GEMM + all-reduce)."""

    @staticmethod
    def forward(ctx, x, weight, group):
        ctx.save_for_backward(x, weight)
        ctx.group = group
        x2 = x.reshape(-1, x.shape[-1])
        return matmul(x2, weight).reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        x2 = x.reshape(-1, x.shape[-1])
        dy2 = aligned_rows(dy.reshape(-1, dy.shape[-1]))
        dx = None
        if ctx.needs_input_grad[0]:
            if tp_fused.usable(dy2, weight.shape[1], ctx.group):
                dx = tp_fused.fused_for(ctx.group, dy2.device)(dy2, aligned_rows(weight), b_mn=True)
            else:
                dx = _sum_over_group(matmul(dy2, weight, b_mn=True), ctx.group)
            dx = dx.reshape(x.shape)
        dw = weight_grad(dy2, x2, weight) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class _RowLinearFused(torch.autograd.Function):
    """y = sum over the group of x_shard W_shard^T (fused GEMM + all-reduce); dx = dy W_shard locally."""

    @staticmethod
    def forward(ctx, x, weight, group):
        ctx.save_for_backward(x, weight)
        x2 = aligned_rows(x.reshape(-1, x.shape[-1]))
        y = tp_fused.fused_for(group, x2.device)(x2, aligned_rows(weight))
        return y.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        x2 = x.reshape(-1, x.shape[-1])
        dy2 = aligned_rows(dy.reshape(-1, dy.shape[-1]))
        dx = matmul(dy2, weight, b_mn=True).reshape(x.shape) if ctx.needs_input_grad[0] else None
        dw = weight_grad(dy2, x2, weight) if ctx.needs_input_grad[1] else None
        return dx, dw, None


def column_linear(x: torch.Tensor, weight: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    if tp is not None and tp.enabled:
        if tp_fused.usable(x, weight.shape[1], tp.group):
            return _ColumnLinearFused.apply(x, weight, tp.group)
        x = _CopyToTP.apply(x, tp.group)
    return linear(x, weight)


def row_linear(x: torch.Tensor, weight: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    if tp is not None and tp.enabled and tp_fused.usable(x, weight.shape[0], tp.group):
        return _RowLinearFused.apply(x, weight, tp.group)
    y = linear(x, weight)
    if tp is not None and tp.enabled:
        y = _ReduceFromTP.apply(y, tp.group)
    return y


def shard_rows(full: torch.Tensor, parts, tp: TPContext | None) -> torch.Tensor:
    """Rows of this TP index from a weight whose rows are the concatenation of ``parts``
    (each part split evenly over the group), e.g. [q | k | v] of a fused projection."""
    if tp is None or not tp.enabled:
        return full
    out, start = [], 0
    for n in parts:
        if n % tp.tp:
            raise ValueError("a sharded projection part must split evenly over the TP group")
        w = n // tp.tp
        out.append(full[start + tp.index * w:start + (tp.index + 1) * w])
        start += n
    if start != full.shape[0]:
        out.append(full[start:][:0])
    return torch.cat(out, 0)


def shard_cols(full: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    if tp is None or not tp.enabled:
        return full
    w = full.shape[1] // tp.tp
    return full[:, tp.index * w:(tp.index + 1) * w]
