"""RoPE, causal short convolution + SiLU, and SwiGLU.

* RoPE: rotate-half rotary embedding with base 10000 applied in place to the
  q/k column blocks of the fused QKV projection; positions are per-token ids
  (zigzag CP chunks carry their true sequence positions), reference
  ``rope_utils.apply_rotary_pos_emb`` with ``cu_seqlens``.
* conv1d: depthwise causal convolution (kernel 4) over the packed q/k/v
  channels of a GDN layer, reset at sequence starts, with an optional 3-token
  halo that carries the previous CP rank's tail of the same sequence.
* SwiGLU: ``silu(a) * b`` over the two halves of fc1's output.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._lib import aligned_rows, is_cuda, lib, on_main_grad


# ---------------------------------------------------------------- RoPE
def _ref_rope(x, pos, heads, d, base, inverse):
    T = x.shape[0]
    xf = x.float().reshape(T, heads, d)
    inv_freq = 1.0 / (base ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    ang = pos.float()[:, None] * inv_freq[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    if inverse:
        sin = -sin
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    out = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)
    return out.reshape(T, heads * d).to(x.dtype)


class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, pos, heads, d, base):
        y = x.contiguous().clone() if x.is_contiguous() else x.contiguous()
        lib().rope_inplace(y, pos, heads, d, base, False)
        ctx.save_for_backward(pos)
        ctx.cfg = (heads, d, base)
        return y

    @staticmethod
    def backward(ctx, dy):
        (pos,) = ctx.saved_tensors
        heads, d, base = ctx.cfg
        dx = dy.contiguous().clone()
        lib().rope_inplace(dx, pos, heads, d, base, True)
        return dx, None, None, None, None


def rope(x: torch.Tensor, positions: torch.Tensor, heads: int, head_dim: int, base: float = 10000.0):
    """Rotary embedding of ``x`` [T, heads*head_dim] at integer ``positions`` [T]."""
    if not is_cuda(x):
        return _ref_rope(x, positions, heads, head_dim, base, False)
    return _Rope.apply(x, positions.to(torch.int32), heads, head_dim, base)


# ---------------------------------------------------------------- conv1d
def _ref_conv(x, w, halo, cu):
    T, C = x.shape
    K = w.shape[1]
    out = torch.empty((T, C), dtype=torch.float32, device=x.device)
    cu_list = cu.tolist()
    for s in range(len(cu_list) - 1):
        a, b = cu_list[s], cu_list[s + 1]
        seg = x[a:b].float()
        if s == 0 and halo is not None:
            pad = halo.float()
        else:
            pad = torch.zeros((K - 1, C), dtype=torch.float32, device=x.device)
        full = torch.cat([pad, seg], 0)  # [(K-1)+n, C]
        y = F.conv1d(full.t()[None], w.float()[:, None, :], groups=C)[0].t()
        out[a:b] = F.silu(y)
    return out.to(x.dtype)


class _Conv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, halo, cu):
        y = lib().conv1d_silu_fwd(x, w, halo, cu)
        ctx.save_for_backward(x, w, halo, cu)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, halo, cu = ctx.saved_tensors
        dx = torch.empty(x.shape, device=x.device, dtype=x.dtype)
        res = lib().conv1d_silu_bwd(dy.contiguous(), x, w, halo, cu, dx)
        dw = res[0]
        main = getattr(w, "main_grad", None)
        if main is not None:
            main.add_(dw)
            dw = None
            on_main_grad(w)
        else:
            dw = dw.to(w.dtype)
        dhalo = res[1].to(halo.dtype) if halo is not None else None
        return dx, dw, dhalo, None


def causal_conv1d_silu(x: torch.Tensor, weight: torch.Tensor, cu_seqlens: torch.Tensor,
                       halo: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(depthwise_causal_conv(x))`` per sequence; ``x`` [T, C], ``weight`` [C, 4]."""
    if not is_cuda(x):
        return _ref_conv(x, weight, halo, cu_seqlens)
    if x.stride(-1) != 1:
        x = x.contiguous()
    return _Conv.apply(x, weight, halo, cu_seqlens.to(torch.int32))


# ---------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        T, F2 = x.shape
        y = torch.empty((T, F2 // 2), device=x.device, dtype=x.dtype)
        lib().swiglu_fwd(x, y)
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dx = torch.empty_like(x)
        lib().swiglu_bwd(dy.contiguous(), x, dx)
        return dx


def swiglu(x: torch.Tensor) -> torch.Tensor:
    """``silu(x[:, :F]) * x[:, F:]`` for ``x`` [T, 2F]."""
    if not is_cuda(x):
        a, b = x.float().chunk(2, dim=-1)
        return (F.silu(a) * b).to(x.dtype)
    return _SwiGLU.apply(aligned_rows(x))
