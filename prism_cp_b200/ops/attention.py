"""Variable-length causal/full GQA attention (THD packing, head_dim 128 on GPU).

``AttentionMeta`` carries one packed layout: the per-sequence query/key lengths
(host ints, known from the plan), the device ``cu_seqlens`` and the work-tile
table of the tcgen05 kernels (longest causal tiles first). Semantics follow
FlashAttention varlen with ``causal`` top-left aligned per sequence, returning
the natural-log LSE ``[heads, tokens]`` so ring (context-parallel) partial
results can be merged exactly.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ._lib import is_cuda, lib, status

TILE = 128


@dataclass
class AttentionMeta:
    q_lens: tuple[int, ...]
    k_lens: tuple[int, ...]
    causal: bool
    device: torch.device
    cu_q: torch.Tensor = field(init=False)
    cu_k: torch.Tensor = field(init=False)
    tiles: torch.Tensor = field(init=False)
    tiles_k: torch.Tensor = field(init=False)

    def __post_init__(self):
        if len(self.q_lens) != len(self.k_lens):
            raise ValueError("query and key sequence counts differ")
        if self.causal and any(a != b for a, b in zip(self.q_lens, self.k_lens)):
            raise ValueError("causal attention requires equal query/key lengths per sequence")
        cq, ck = [0], [0]
        for a, b in zip(self.q_lens, self.k_lens):
            cq.append(cq[-1] + a)
            ck.append(ck[-1] + b)
        self.cu_q = torch.tensor(cq, dtype=torch.int32, device=self.device)
        self.cu_k = torch.tensor(ck, dtype=torch.int32, device=self.device)
        # forward tiles: (seq, q tile), heaviest first
        work = []
        for s, (lq, lk) in enumerate(zip(self.q_lens, self.k_lens)):
            for t in range((lq + TILE - 1) // TILE):
                kv = min(lk, (t + 1) * TILE) if self.causal else lk
                work.append((-kv, s, t))
        work.sort()
        rows = [(s, t) for _, s, t in work] or [(0, 0)]
        self.tiles = torch.tensor(rows[: len(work)] if work else [], dtype=torch.int32,
                                  device=self.device).reshape(-1, 2)
        # backward tiles: (seq, kv tile), heaviest first
        work = []
        for s, (lq, lk) in enumerate(zip(self.q_lens, self.k_lens)):
            for t in range((lk + TILE - 1) // TILE):
                q = lq - t * TILE if self.causal else lq
                work.append((-q, s, t))
        work.sort()
        self.tiles_k = torch.tensor([(s, t) for _, s, t in work], dtype=torch.int32,
                                    device=self.device).reshape(-1, 2)

    @property
    def total_q(self):
        return sum(self.q_lens)

    @property
    def total_k(self):
        return sum(self.k_lens)


def reference_attention(q, k, v, meta: AttentionMeta, scale: float):
    """fp32 PyTorch oracle: returns (out [Tq,Hq,d], lse [Hq,Tq])."""
    Tq, Hq, d = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    out = torch.zeros((Tq, Hq, d), dtype=torch.float32, device=q.device)
    lse = torch.full((Hq, Tq), float("-inf"), dtype=torch.float32, device=q.device)
    oq = ok = 0
    for lq, lk in zip(meta.q_lens, meta.k_lens):
        qs = q[oq:oq + lq].float().transpose(0, 1)                       # [Hq, lq, d]
        ks = k[ok:ok + lk].float().transpose(0, 1).repeat_interleave(rep, 0)
        vs = v[ok:ok + lk].float().transpose(0, 1).repeat_interleave(rep, 0)
        s = qs @ ks.transpose(1, 2) * scale
        if meta.causal:
            mask = torch.ones((lq, lk), dtype=torch.bool, device=q.device).tril()
            s = s.masked_fill(~mask, float("-inf"))
        m = torch.logsumexp(s, dim=-1)                                   # [Hq, lq]
        p = torch.exp(s - m[..., None])
        out[oq:oq + lq] = (p @ vs).transpose(0, 1)
        lse[:, oq:oq + lq] = m
        oq += lq
        ok += lk
    return out.to(q.dtype), lse


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, meta, scale):
        out = torch.empty((q.shape[0], q.shape[1], q.shape[2]), device=q.device, dtype=q.dtype)
        lse = torch.empty((q.shape[1], q.shape[0]), device=q.device, dtype=torch.float32)
        lib().attention_fwd(q, k, v, meta.cu_q, meta.cu_k, meta.tiles, out, lse, meta.causal, scale,
                            status(q.device))
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.meta, ctx.scale = meta, scale
        return out, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = attention_backward(q, k, v, out, lse, dout, ctx.meta, ctx.scale)
        return dq, dk, dv, None, None


def reference_attention_backward(q, k, v, out, lse, dout, meta: AttentionMeta, scale: float):
    """fp32 oracle of the flash backward given the (possibly ring-merged) out and LSE."""
    Tq, Hq, d = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    dk = torch.zeros(k.shape, dtype=torch.float32, device=k.device)
    dv = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
    oq = ok = 0
    for lq, lk in zip(meta.q_lens, meta.k_lens):
        qs = q[oq:oq + lq].float().transpose(0, 1)
        ks = k[ok:ok + lk].float().transpose(0, 1).repeat_interleave(rep, 0)
        vs = v[ok:ok + lk].float().transpose(0, 1).repeat_interleave(rep, 0)
        do = dout[oq:oq + lq].float().transpose(0, 1)
        o = out[oq:oq + lq].float().transpose(0, 1)
        s = qs @ ks.transpose(1, 2) * scale
        if meta.causal:
            mask = torch.ones((lq, lk), dtype=torch.bool, device=q.device).tril()
            s = s.masked_fill(~mask, float("-inf"))
        p = torch.nan_to_num(torch.exp(s - lse[:, oq:oq + lq, None]), nan=0.0)
        dvs = p.transpose(1, 2) @ do
        dp = do @ vs.transpose(1, 2)
        ds = p * (dp - (do * o).sum(-1, keepdim=True))
        dq[oq:oq + lq] = (ds @ ks * scale).transpose(0, 1)
        dk[ok:ok + lk] = (ds.transpose(1, 2) @ qs * scale).reshape(Hkv, rep, lk, d).sum(1).transpose(0, 1)
        dv[ok:ok + lk] = dvs.reshape(Hkv, rep, lk, d).sum(1).transpose(0, 1)
        oq += lq
        ok += lk
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def attention_backward(q, k, v, out, lse, dout, meta, scale):
    """Flash backward from the (global) out/LSE; the tcgen05 kernels on CUDA."""
    if not is_cuda(q):
        return reference_attention_backward(q, k, v, out, lse, dout, meta, scale)
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dkv = torch.empty((k.shape[0], 2, k.shape[1], k.shape[2]), device=k.device, dtype=k.dtype)
    dk, dv = dkv[:, 0], dkv[:, 1]
    lib().attention_bwd(q, k, v, out, lse, dout.contiguous(), meta.cu_q, meta.cu_k, meta.tiles, meta.tiles_k,
                        dq, dk, dv, meta.causal, scale, status(q.device))
    return dq, dk, dv


def flash_attention(q, k, v, meta: AttentionMeta, scale: float | None = None):
    """Return ``(out, lse)`` for ``q`` [Tq,Hq,d], ``k``/``v`` [Tk,Hkv,d]."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    if not is_cuda(q):
        return _RefAttention.apply(q, k, v, meta, scale)
    return _FlashAttention.apply(q, k, v, meta, scale)


class _RefAttention(torch.autograd.Function):
    """CPU path with an explicit backward that matches the kernel's math."""

    @staticmethod
    def forward(ctx, q, k, v, meta, scale):
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            o, lse = reference_attention(qq, kk, vv, meta, scale)
        ctx.saved = (qq, kk, vv, o, lse)
        return o.detach(), lse.detach()

    @staticmethod
    def backward(ctx, dout, dlse):
        qq, kk, vv, o, lse = ctx.saved
        outs, grads = [o], [dout]
        if dlse is not None:
            outs.append(lse)
            grads.append(dlse)
        dq, dk, dv = torch.autograd.grad(outs, (qq, kk, vv), grads, allow_unused=True)
        return dq, dk, dv, None, None
