"""RMSNorm, gated RMSNorm (GDN output norm) and per-head L2 norm.

All three are the same row operation ``y = x * rsqrt(inv_n * sum(x^2) + eps)
[* w] [* silu(z)]`` and share one CUDA kernel family (``csrc/norms.cu``).
Reference semantics: Megatron ``--normalization RMSNorm`` (pre-norm, eps 1e-6 by
default here), the GDN gated output norm and FLA's ``use_qk_l2norm_in_kernel``.
"""

from __future__ import annotations

import torch

from ._lib import aligned_rows, is_cuda, lib, on_main_grad


def _ref_rownorm(x, w, z, heads, n, inv_n, eps):
    shape = x.shape
    xf = x.float().reshape(shape[0], heads, n)
    r = torch.rsqrt(xf.pow(2).sum(-1, keepdim=True) * inv_n + eps)
    y = xf * r
    if w is not None:
        y = y * w.float()
    if z is not None:
        zf = z.float().reshape(shape[0], heads, n)
        y = y * torch.nn.functional.silu(zf)
    return y.reshape(shape[0], heads * n).to(x.dtype)


class _RowNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, z, heads, n, inv_n, eps):
        T = x.shape[0]
        y = torch.empty((T, heads * n), device=x.device, dtype=x.dtype)
        rstd = torch.empty((T * heads,), device=x.device, dtype=torch.float32)
        lib().rownorm_fwd(x, w, z, y, rstd, heads, n, inv_n, eps)
        ctx.save_for_backward(x, w, z, rstd)
        ctx.cfg = (heads, n, inv_n)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, z, rstd = ctx.saved_tensors
        heads, n, inv_n = ctx.cfg
        dy = dy.contiguous()
        dx = torch.empty((x.shape[0], heads * n), device=x.device, dtype=x.dtype)
        dz = torch.empty_like(dx) if z is not None else None
        dw = lib().rownorm_bwd(dy, x, w, z, rstd, dx, dz, heads, n, inv_n)
        if dw is not None:
            main = getattr(w, "main_grad", None)
            if main is not None:
                main.add_(dw)
                dw = None
                on_main_grad(w)
            else:
                dw = dw.to(w.dtype)
        return dx, dw, dz, None, None, None, None


def _rownorm(x, w, z, heads, n, inv_n, eps):
    if not is_cuda(x):
        return _ref_rownorm(x, w, z, heads, n, inv_n, eps)
    x = aligned_rows(x)
    if z is not None:
        z = aligned_rows(z)
    return _RowNorm.apply(x, w, z, heads, n, inv_n, eps)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    shape = x.shape
    h = shape[-1]
    y = _rownorm(x.reshape(-1, h), weight, None, 1, h, 1.0 / h, eps)
    return y.reshape(shape)


def gated_rms_norm(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, heads: int,
                   eps: float = 1e-6) -> torch.Tensor:
    """Per-head RMSNorm of ``x`` [T, heads*n] times ``weight`` [n] times ``silu(gate)``."""
    n = x.shape[-1] // heads
    return _rownorm(x, weight, gate, heads, n, 1.0 / n, eps)


def l2_norm(x: torch.Tensor, heads: int, eps: float = 1e-6) -> torch.Tensor:
    """Per-head ``x / sqrt(sum(x^2) + eps)`` over rows of ``x`` [T, heads*n]."""
    n = x.shape[-1] // heads
    return _rownorm(x, None, None, heads, n, 1.0, eps)
