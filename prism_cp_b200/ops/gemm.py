"""Matrix products on the tcgen05 GEMM and the linear layer built on it.

``matmul(a, b)`` computes ``C[m, n] = sum_k A(m, k) B(n, k)`` where ``a`` is
``[M, K]`` (K-major) or ``[K, M]`` (``a_mn=True``) and ``b`` is ``[N, K]`` or
``[K, N]`` (``b_mn=True``). The three GEMMs of a linear layer therefore need no
transposes: forward ``x W^T`` (K/K), input gradient ``dy W`` (K/MN) and weight
gradient ``dy^T x`` (MN/MN), the latter accumulated in fp32 into ``main_grad``
(gradient-accumulation fusion, as Megatron's ``--gradient-accumulation-fusion``).
"""

from __future__ import annotations

import torch

from ._lib import aligned_rows, is_cuda, lib, status, on_main_grad


def _torch_mm(a, b, a_mn, b_mn):
    A = a.t() if a_mn else a
    B = b if b_mn else b.t()
    return A.float() @ B.float()


def matmul(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False,
           out: torch.Tensor | None = None, accumulate: bool = False,
           row_scale: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if not is_cuda(a, b):
        result = _torch_mm(a, b, a_mn, b_mn)
        if row_scale is not None:
            result = result * row_scale[:, None]
        if out is None:
            return result.to(out_dtype or a.dtype)
        if accumulate:
            out.add_(result.to(out.dtype))
        else:
            out.copy_(result)
        return out
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=out_dtype or torch.bfloat16)
    a, b = aligned_rows(a), aligned_rows(b)
    lib().gemm(a, b, out, a_mn, b_mn, accumulate, row_scale, status(a.device))
    return out


def weight_grad(dy2: torch.Tensor, x2: torch.Tensor, weight: torch.Tensor):
    """dW = dy^T x: accumulated in fp32 into ``weight.main_grad`` when it exists (returns None), else returned."""
    main = getattr(weight, "main_grad", None)
    if main is not None and x2.is_cuda:
        matmul(dy2, x2, a_mn=True, b_mn=True, out=main, accumulate=True)
        on_main_grad(weight)
        return None
    if main is not None:
        main.add_(_torch_mm(dy2, x2, True, True).to(main.dtype))
        on_main_grad(weight)
        return None
    return matmul(dy2, x2, a_mn=True, b_mn=True, out_dtype=weight.dtype)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight):
        ctx.save_for_backward(x, weight)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y = matmul(x2, weight)
        return y.reshape(*shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        dy2 = dy.reshape(-1, dy.shape[-1])
        if dy2.stride(-1) != 1:
            dy2 = dy2.contiguous()
        dx = matmul(dy2, weight, b_mn=True).reshape(shape) if ctx.needs_input_grad[0] else None
        dw = weight_grad(dy2, x2, weight) if ctx.needs_input_grad[1] else None
        return dx, dw


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """y = x W^T (no bias). If ``weight.main_grad`` exists, dW accumulates there in fp32."""
    return _Linear.apply(x, weight)
