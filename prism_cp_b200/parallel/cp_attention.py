"""Zigzag ring attention over a CP team (causal GQA, varlen packs).

Rank ``i`` of a team of size ``c`` holds, for every sample of length ``L``, the
chunks ``i`` and ``2c-1-i`` of length ``L / 2c`` (zigzag balances causal work).
KV blocks travel around the ring; at ring step ``t`` rank ``i`` holds the KV of
rank ``j = (i - t) mod c`` and, per sample:
  * ``t = 0``: causal attention over its own two chunks (their concatenation is
    position-ordered, so index-causal masking is exact);
  * ``j < i``: every local query sees only the first KV chunk ``j`` (full);
  * ``j > i``: only the second local query chunk ``2c-1-i`` sees both KV
    chunks (full).
Partial results are merged with their log-sum-exp. The backward repeats the
ring with the merged output and LSE (so every step's P is the globally
normalised probability) and passes each KV block's dK/dV accumulator along
with it, so after ``c`` hops it arrives back at its owner. In both directions
the send/receive of the next block is issued before the current block's
kernels run, so the exchange overlaps the attention kernels.

Reference behaviour: TransformerEngine ``cp_comm_type=p2p`` ring with zigzag
(``attn_forward_func_with_cp``) as driven by the reference's launcher.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.attention import AttentionMeta, attention_backward, flash_attention


def merge_partial(out, lse, o_new, lse_new, rows=None):
    """Merge a partial attention result (o_new [t,H,d], lse_new [H,t]) into out/lse
    (all rows, or the given row indices) with log-sum-exp weights."""
    if rows is None:
        cur_o, cur_l = out, lse
    else:
        cur_o, cur_l = out.index_select(0, rows), lse.index_select(1, rows)
    m = torch.maximum(cur_l, lse_new)
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    a = torch.exp(cur_l - m_safe)
    b = torch.exp(lse_new - m_safe)
    s = a + b
    merged_l = torch.where(s > 0, m_safe + torch.log(s), torch.full_like(s, float("-inf")))
    wa = torch.nan_to_num(a / s).transpose(0, 1)[..., None]
    wb = torch.nan_to_num(b / s).transpose(0, 1)[..., None]
    merged_o = (cur_o.float() * wa + o_new.float() * wb).to(out.dtype)
    if rows is None:
        return merged_o, merged_l
    return out.index_copy(0, rows, merged_o), lse.index_copy(1, rows, merged_l)


class Ring:
    """Static per-layout geometry of the zigzag ring for one rank."""

    def __init__(self, ctx):
        self.c, self.i = ctx.cp, ctx.index
        self.team = ctx.team
        self.ranks = ctx.global_ranks
        lens = [ctx.lengths[s] for s in ctx.samples]
        self.half = [n // (2 * self.c) for n in lens]
        dev = ctx.device
        first, second = [], []
        off = 0
        for h in self.half:
            first.extend(range(off, off + h))
            second.extend(range(off + h, off + 2 * h))
            off += 2 * h
        self.first = torch.tensor(first, dtype=torch.int64, device=dev)
        self.second = torch.tensor(second, dtype=torch.int64, device=dev)
        two = tuple(2 * h for h in self.half)
        self.meta_diag = AttentionMeta(two, two, True, dev)
        self.meta_low = AttentionMeta(two, tuple(self.half), False, dev)    # all q vs first kv chunk
        self.meta_high = AttentionMeta(tuple(self.half), two, False, dev)   # second q chunk vs all kv
        self.next = self.ranks[(self.i + 1) % self.c]
        self.prev = self.ranks[(self.i - 1) % self.c]

    def exchange(self, send: torch.Tensor, recv: torch.Tensor):
        ops = [dist.P2POp(dist.isend, send, self.next, group=self.team),
               dist.P2POp(dist.irecv, recv, self.prev, group=self.team)]
        return dist.batch_isend_irecv(ops)

    def step_kind(self, t: int) -> str:
        j = (self.i - t) % self.c
        return "diag" if t == 0 else ("low" if j < self.i else "high")


class _ZigzagRingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, ring: Ring, scale):
        T, H, d = q.shape
        cur = torch.stack([k, v]).contiguous()
        out = torch.zeros((T, H, d), dtype=q.dtype, device=q.device)
        lse = torch.full((H, T), float("-inf"), dtype=torch.float32, device=q.device)
        for t in range(ring.c):
            reqs, nxt = None, None
            if t + 1 < ring.c:
                nxt = torch.empty_like(cur)
                reqs = ring.exchange(cur, nxt)
            kind = ring.step_kind(t)
            kk, vv = cur[0], cur[1]
            if kind == "diag":
                out, lse = flash_attention(q, kk, vv, ring.meta_diag, scale)
            elif kind == "low":
                o, l = flash_attention(q, kk.index_select(0, ring.first), vv.index_select(0, ring.first),
                                       ring.meta_low, scale)
                out, lse = merge_partial(out, lse, o, l)
            else:
                o, l = flash_attention(q.index_select(0, ring.second), kk, vv, ring.meta_high, scale)
                out, lse = merge_partial(out, lse, o, l, ring.second)
            if reqs is not None:
                for r in reqs:
                    r.wait()
                cur = nxt
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.ring, ctx.scale = ring, scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        ring, scale = ctx.ring, ctx.scale
        dout = dout.contiguous()
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        kv = torch.stack([k, v]).contiguous()
        sec = ring.second
        q2, o2, do2, lse2 = q.index_select(0, sec), out.index_select(0, sec), dout.index_select(0, sec), \
            lse.index_select(1, sec)
        # Both exchanges overlap the kernels: the next KV block is requested before this step's
        # kernels run, and the dK/dV accumulator of the block that arrives next is received while
        # this step computes its own contribution, which is added when the accumulator lands.
        acc_req = acc_in = None
        for t in range(ring.c):
            kv_req = nkv = None
            if t + 1 < ring.c:
                nkv = torch.empty_like(kv)
                kv_req = ring.exchange(kv, nkv)
            kind = ring.step_kind(t)
            kk, vv = kv[0], kv[1]
            part = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)
            if kind == "diag":
                a, b, c = attention_backward(q, kk, vv, out, lse, dout, ring.meta_diag, scale)
                dq += a.float()
                part[0] += b.float()
                part[1] += c.float()
            elif kind == "low":
                kf, vf = kk.index_select(0, ring.first), vv.index_select(0, ring.first)
                a, b, c = attention_backward(q, kf, vf, out, lse, dout, ring.meta_low, scale)
                dq += a.float()
                part[0].index_add_(0, ring.first, b.float())
                part[1].index_add_(0, ring.first, c.float())
            else:
                a, b, c = attention_backward(q2, kk, vv, o2, lse2, do2, ring.meta_high, scale)
                dq.index_add_(0, sec, a.float())
                part[0] += b.float()
                part[1] += c.float()
            if acc_req is not None:
                for r in acc_req:
                    r.wait()
                part += acc_in
            # the accumulator follows its KV block around the ring and finally returns to the owner
            acc_in = torch.empty_like(part)
            acc_req = ring.exchange(part, acc_in)
            if kv_req is not None:
                for r in kv_req:
                    r.wait()
                kv = nkv
        for r in acc_req:
            r.wait()
        dkv = acc_in
        return dq.to(q.dtype), dkv[0].to(k.dtype), dkv[1].to(v.dtype), None, None


class ZigzagRing:
    def __init__(self, ctx):
        self.ring = Ring(ctx)

    def __call__(self, q, k, v, scale=None):
        scale = q.shape[-1] ** -0.5 if scale is None else scale
        return _ZigzagRingFn.apply(q, k, v, self.ring, scale)
