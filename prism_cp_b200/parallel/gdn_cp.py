"""Gated-DeltaNet context parallelism over a contiguous layout.

The team's packed samples are sliced evenly across its ranks, so a rank's first
local segment may continue a sample from the previous rank and its last segment
may continue on the next one. Two things cross ranks:

* conv halo - the 3 tokens before a continuing segment, sent by the previous
  rank (forward) with the matching gradient sent back (backward);
* recurrent state - the state a continuing sample carries into this rank.
  Every rank runs a zero-start state pass over its last segment only (the one
  that continues on the next rank), giving that segment's final state ``F``,
  and, when one sample spans the whole rank, the tail's transition matrix
  ``M`` (``S_out = M S_in + F``).
  ``(F, M)`` are all-gathered over the team (differentiable), each rank folds
  the prefix of its chain of predecessors and then runs the real state pass
  from that state. Forward and backward are parallel across the team (no rank
  waits for another rank's recurrence); gradients reach the predecessors' ``F``
  and ``M`` through the all-gather's backward.

Reference behaviour: Megatron GDN ``--linear-cp-mode chunkwise`` with the
state exchange modelled at joint_cp/model.py:141-145.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.elementwise import causal_conv1d_silu
from ..ops.gdn import (chunk_output, chunk_prep, chunk_state, chunk_transition, fused_gated_delta_rule,
                       fused_supported)
from ..planner.joint.ir import spans as layout_spans

HALO = 3


class _Tie(torch.autograd.Function):
    """Identity on ``x`` that also makes ``anchor`` part of the graph.

    A collective's backward must run on every rank of the team, but a rank that
    does not consume the collective's result would otherwise drop it from its
    graph. Tying the result to the layer output (with a zero gradient) keeps the
    backward collectives matched on all ranks.
    """

    @staticmethod
    def forward(ctx, x, anchor):
        ctx.anchor_shape, ctx.anchor_dtype = anchor.shape, anchor.dtype
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        return grad, torch.zeros(ctx.anchor_shape, dtype=ctx.anchor_dtype, device=grad.device)


def tie(x, anchor):
    return _Tie.apply(x, anchor)


class _AllGather(torch.autograd.Function):
    """All-gather of equal-size flat tensors over a team; the backward sums every
    rank's gradient of the stacked result and keeps this rank's row (group-relative
    ranks throughout, so it works for teams of any global ranks)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        out = [torch.empty_like(x) for _ in range(n)]
        dist.all_gather(out, x.contiguous(), group=group)
        return torch.stack(out)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g[dist.get_rank(ctx.group)], None


def all_gather_rows(x, group):
    return _AllGather.apply(x, group)


def rank_links(ctx):
    """Per team rank: (first segment continues from prev, last continues to next, single segment)."""
    rows = layout_spans(ctx.layout, ctx.lengths, ctx.world)
    out = []
    for r in ctx.group_ranks:
        row = rows[r]
        if not row:
            out.append((False, False, False))
            continue
        _, b0, _, _ = row[0]
        sl, bl, _, cl = row[-1]
        out.append((b0 > 0, bl + cl < ctx.lengths[sl], len(row) == 1))
    return out


class _HaloExchange(torch.autograd.Function):
    """Forward: send my last rows to the next rank, receive the previous rank's.
    Backward: send the halo gradient back and receive the next rank's."""

    @staticmethod
    def forward(ctx, tail, prev_rank, next_rank, has_prev, has_next, group):
        ctx.cfg = (prev_rank, next_rank, has_prev, has_next, group)
        recv = torch.zeros(tail.shape, dtype=tail.dtype, device=tail.device)
        ops = []
        if has_next:
            ops.append(dist.P2POp(dist.isend, tail.contiguous(), next_rank, group=group))
        if has_prev:
            ops.append(dist.P2POp(dist.irecv, recv, prev_rank, group=group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        return recv

    @staticmethod
    def backward(ctx, grad):
        prev_rank, next_rank, has_prev, has_next, group = ctx.cfg
        out = torch.zeros(grad.shape, dtype=grad.dtype, device=grad.device)
        ops = []
        if has_prev:
            ops.append(dist.P2POp(dist.isend, grad.contiguous(), prev_rank, group=group))
        if has_next:
            ops.append(dist.P2POp(dist.irecv, out, next_rank, group=group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        return out, None, None, None, None, None


def conv_with_halo(ctx, x, weight):
    links = rank_links(ctx)
    i, c = ctx.index, ctx.cp
    first_cont = links[i][0]
    has_next = i + 1 < c and links[i + 1][0]
    if x.shape[0] >= HALO:
        tail = x[-HALO:]
    else:
        tail = torch.cat([x.new_zeros((HALO - x.shape[0], x.shape[1])), x], 0)
    prev_rank = ctx.global_ranks[i - 1] if i > 0 else -1
    next_rank = ctx.global_ranks[i + 1] if i + 1 < c else -1
    halo = _HaloExchange.apply(tail, prev_rank, next_rank, first_cont, has_next, ctx.team)
    if not first_cont:
        return tie(causal_conv1d_silu(x, weight, ctx.cu_segments), halo)
    begin = ctx.spans[0][1]
    if begin < HALO:  # the sample started fewer than 3 tokens before this rank
        keep = torch.zeros((HALO, 1), dtype=halo.dtype, device=halo.device)
        keep[HALO - begin:] = 1
        halo = halo * keep
    return causal_conv1d_silu(x, weight, ctx.cu_segments, halo)


def delta_rule_cp(ctx, q, k, v, g, beta):
    layout = ctx.chunk_layout()
    links = rank_links(ctx)
    i = ctx.index
    first_cont, last_cont, single = links[i]
    H, DK, DV = q.shape[1], q.shape[2], v.shape[2]
    nseg = len(ctx.segment_lengths)
    f32 = torch.float32
    fused = fused_supported(q, v)
    prep = None if fused else chunk_prep(q, k, v, g, beta, layout)
    if fused and last_cont:
        # tail state from zero, and (for a single continuing segment) the linear
        # map of the incoming state: the recurrence with zero values from I
        # these passes only feed a small state: recomputed in the backward rather than kept
        n_last = ctx.segment_lengths[-1]
        if nseg > 1 and n_last >= 64:
            # only the last segment continues on the next rank: run the tail pass over its rows alone
            if getattr(ctx, "_tail_layout", None) is None:
                from ..ops.gdn import ChunkLayout
                ctx._tail_layout = ChunkLayout((n_last,), q.device)
            rows = slice(q.shape[0] - n_last, None)
            _, S_last = fused_gated_delta_rule(q[rows], k[rows], v[rows], g[rows], beta[rows], ctx._tail_layout,
                                               keep_intermediates=False)
            F_tail = S_last[0]
        else:
            _, S_zero = fused_gated_delta_rule(q, k, v, g, beta, layout, keep_intermediates=False)
            F_tail = S_zero[nseg - 1]
        if first_cont and single:
            eye = torch.eye(DK, dtype=f32, device=q.device).expand(nseg, H, DK, DK).contiguous()
            _, M_all = fused_gated_delta_rule(q, k, torch.zeros_like(q), g, beta, layout, initial_state=eye,
                                              keep_intermediates=False)
            M_tail = M_all[nseg - 1]
        else:
            M_tail = torch.zeros((H, DK, DK), dtype=f32, device=q.device)
    elif fused:
        F_tail = torch.zeros((H, DK, DV), dtype=f32, device=q.device)
        M_tail = torch.zeros((H, DK, DK), dtype=f32, device=q.device)
    elif last_cont:
        _, _, S_zero = chunk_state(prep, None)
        F_tail = S_zero[nseg - 1]
        if first_cont and single:
            M_tail = chunk_transition(prep, nseg - 1)
        else:
            M_tail = torch.zeros((H, DK, DK), dtype=f32, device=q.device)
    else:
        F_tail = torch.zeros((H, DK, DV), dtype=f32, device=q.device)
        M_tail = torch.zeros((H, DK, DK), dtype=f32, device=q.device)
    packed = torch.cat([F_tail.reshape(-1), M_tail.reshape(-1)])
    if torch.is_grad_enabled() and not packed.requires_grad:
        # a rank whose contribution is a constant must still own an all-gather
        # backward node, or the team's backward collectives would not match
        packed = packed.detach().requires_grad_(True)
    gathered = all_gather_rows(packed, ctx.team)
    initial = None
    if first_cont:
        chain = [i - 1]
        while chain[-1] > 0 and links[chain[-1]][0] and links[chain[-1]][2]:
            chain.append(chain[-1] - 1)

        def unpack(r):
            t = gathered[r]
            return t[:H * DK * DV].view(H, DK, DV), t[H * DK * DV:].view(H, DK, DK)

        state = unpack(chain[-1])[0]
        for r in reversed(chain[:-1]):
            F_r, M_r = unpack(r)
            state = M_r @ state + F_r
        rest = torch.zeros((nseg - 1, H, DK, DV), dtype=f32, device=q.device)
        initial = torch.cat([state[None], rest], 0)
    if fused:
        o, _ = fused_gated_delta_rule(q, k, v, g, beta, layout, initial_state=initial)
        return tie(o, gathered)
    Delta, S_all, _ = chunk_state(prep, initial)
    return tie(chunk_output(prep, Delta, S_all), gathered)
