"""Column split whose backward writes the input gradient once.

Slicing a projection output into several operands (``p[:, a:b]``) makes
autograd build the input gradient from one zero-filled full-size tensor per
slice plus as many additions. ``split_columns`` returns the same views, and its
backward concatenates the operand gradients into one freshly written tensor
(zeros only for operands that received no gradient).
"""

from __future__ import annotations

import torch


class _SplitColumns(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, sizes):
        ctx.sizes = sizes
        ctx.shape, ctx.dtype, ctx.device = x.shape, x.dtype, x.device
        outs, start = [], 0
        for n in sizes:
            outs.append(x.narrow(-1, start, n))
            start += n
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        parts = []
        lead = ctx.shape[:-1]
        for g, n in zip(grads, ctx.sizes):
            parts.append(g.to(ctx.dtype) if g is not None else torch.zeros(lead + (n,), dtype=ctx.dtype,
                                                                            device=ctx.device))
        rest = ctx.shape[-1] - sum(ctx.sizes)
        if rest:
            parts.append(torch.zeros(lead + (rest,), dtype=ctx.dtype, device=ctx.device))
        return torch.cat(parts, dim=-1), None


def split_columns(x: torch.Tensor, sizes) -> tuple:
    """Views ``x[..., a_i:a_i + sizes[i]]`` (consecutive from 0) with a single-write backward."""
    return _SplitColumns.apply(x, tuple(int(n) for n in sizes))
