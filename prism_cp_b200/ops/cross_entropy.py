"""Untied output head fused with per-token cross-entropy.

The logits of a token chunk are produced by the tcgen05 GEMM, the fused CE
kernel turns them in place into ``weight * (softmax - onehot)`` while writing
the per-token loss, and the two gradient GEMMs consume them immediately, so
the full ``[tokens, vocab]`` logit matrix never exists and no logit is read
twice from HBM after the softmax pass. The loss is ``sum_t weight_t * ce_t``;
with ``weight = loss_mask / loss_tokens`` this is Megatron's per-token loss
(``--calculate-per-token-loss``) normalised over the update.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._lib import is_cuda, lib, on_main_grad
from .gemm import matmul

CHUNK_TOKENS = 8192


class _HeadCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, labels, token_weight, chunk):
        T, H = h.shape
        V = weight.shape[0]
        dh = torch.empty_like(h)
        dw = torch.zeros((V, H), device=h.device, dtype=torch.float32)
        ce = torch.empty((T,), device=h.device, dtype=torch.float32)
        logits = torch.empty((min(chunk, T), V), device=h.device, dtype=torch.bfloat16)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            lg = logits[: e - s]
            matmul(h[s:e], weight, out=lg)
            lib().ce_fused(lg, labels[s:e], token_weight[s:e], ce[s:e], None)
            matmul(lg, weight, b_mn=True, out=dh[s:e])
            matmul(lg, h[s:e], a_mn=True, b_mn=True, out=dw, accumulate=True)
        ctx.save_for_backward(dh, dw)
        ctx.weight = weight
        loss = (ce * token_weight).sum()
        ctx.mark_non_differentiable(ce)
        return loss, ce

    @staticmethod
    def backward(ctx, g, _unused):
        dh, dw = ctx.saved_tensors
        weight = ctx.weight
        main = getattr(weight, "main_grad", None)
        if main is not None:
            main.addcmul_(dw, g.to(torch.float32).reshape(1, 1))
            dweight = None
            on_main_grad(weight)
        else:
            dweight = (dw * g).to(weight.dtype)
        return (dh * g.to(dh.dtype)), dweight, None, None, None


def head_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                       token_weight: torch.Tensor, chunk: int = CHUNK_TOKENS):
    """Return ``(loss, ce)``: weighted loss sum and per-token CE (no grad)."""
    if not is_cuda(h):
        logits = h.float() @ weight.float().t()
        ce = F.cross_entropy(logits, labels, reduction="none")
        return (ce * token_weight).sum(), ce.detach()
    return _HeadCE.apply(h.contiguous(), weight, labels.to(torch.int64), token_weight.float().contiguous(), chunk)
