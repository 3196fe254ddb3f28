"""Gated-DeltaNet context parallelism over a contiguous layout.

The team's packed samples are sliced evenly across its ranks, so a rank's first
local segment may continue a sample from the previous rank and its last segment
may continue on the next one. Two things cross ranks:

* conv halo - the 3 tokens before a continuing segment, sent by the previous
  rank (forward) with the matching gradient sent back (backward);
* recurrent state - the state a continuing sample carries into this rank.
  The recurrence is affine in that state, so every rank runs its segments from
  zero (outputs and the last segment's final state ``F``) and, when its first
  segment continues a sample, the zero-value recurrence of that segment from
  the identity (per-token rows ``L`` and the transition matrix ``M``,
  ``S_out = M S_in + F``) on a second stream. ``(F, M)`` are all-gathered over
  the team (differentiable), each rank folds the prefix of its chain of
  predecessors into ``S_in`` and adds ``L S_in`` to its first segment's
  outputs. Forward and backward are parallel across the team (no rank waits
  for another rank's recurrence); gradients reach the predecessors' ``F`` and
  ``M`` through the all-gather's backward.

Reference behaviour: Megatron GDN ``--linear-cp-mode chunkwise`` with the
state exchange modelled at joint_cp/model.py:141-145.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops.elementwise import causal_conv1d_silu
from ..ops.gdn import chunk_gated_delta_rule, fused_affine_delta_rule, fused_gated_delta_rule, fused_supported
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


_SIDE: dict = {}
# PRISM_GDN_SHARED_PREP=1: both passes of a continuing rank on one prep and one local backward
# (``ops.gdn.fused_affine_delta_rule``); the default runs them as two fused rules on two streams
SHARED_PREP = os.environ.get("PRISM_GDN_SHARED_PREP", "0") == "1"


def _side_stream(device) -> torch.cuda.Stream:
    s = _SIDE.get(device.index)
    if s is None:
        s = _SIDE[device.index] = torch.cuda.Stream(device=device)
    return s


def _rule(q, k, v, g, beta, layout, initial_state=None):
    """(o, per-segment final states) on the fused kernels where they apply, else the chunked torch form."""
    if fused_supported(q, v):
        return fused_gated_delta_rule(q, k, v, g, beta, layout, initial_state=initial_state)
    return chunk_gated_delta_rule(q, k, v, g, beta, layout, initial_state=initial_state)


def _first_layout(ctx, layout, nseg: int, n0: int):
    if nseg == 1:
        return layout
    if getattr(ctx, "_first_layout", None) is None:
        from ..ops.gdn import ChunkLayout
        ctx._first_layout = ChunkLayout((n0,), layout.tok0_dev.device)
    return ctx._first_layout


def _identity_pass(q, k, g, beta, n0: int, lay0):
    """(L, M) of the first segment by a separate zero-value rule from the identity (a second CUDA
    stream next to the caller's; the torch form on CPU)."""
    H, DK = q.shape[1], q.shape[2]

    def run():
        eye = torch.eye(DK, dtype=torch.float32, device=q.device).expand(1, H, DK, DK).contiguous()
        return _rule(q[:n0], k[:n0], q.new_zeros((n0, H, DK)), g[:n0], beta[:n0], lay0, initial_state=eye)

    if not q.is_cuda:
        return run()
    main, side = torch.cuda.current_stream(q.device), _side_stream(q.device)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        out = run()
    for t in (q, k, g, beta):
        t.record_stream(side)
    return out


def delta_rule_cp(ctx, q, k, v, g, beta):
    """The recurrence of this rank's segments, with the state a continuing sample carries in.

    The recurrence is affine in the incoming state S_in of the first segment: every output row is
    o_t = o0_t + L_t S_in and the segment's final state is F + M S_in, where o0 and F come from the
    pass started at zero and L (one dk-row per token and head) and M from the same recurrence with
    zero values started at the identity. So each rank runs
      * the zero-start pass over all its segments (outputs, and F of the last segment), and
      * if its first segment continues a sample, the zero-value pass over that segment alone
        (dv = dk, on a second stream, concurrently with the first); with PRISM_GDN_SHARED_PREP=1
        both passes share one prep and one local backward (``ops.gdn.fused_affine_delta_rule``),
    all-gathers (F, M) of its last segment over the team, folds its predecessors' chain into S_in
    and adds L S_in to the first segment's rows: no pass waits for another rank, and no pass is run
    twice. Gradients reach both passes and the predecessors' (F, M) through autograd and the
    all-gather's backward.
    """
    layout = ctx.chunk_layout()
    links = rank_links(ctx)
    i = ctx.index
    first_cont, last_cont, single = links[i]
    H, DK, DV = q.shape[1], q.shape[2], v.shape[2]
    nseg = len(ctx.segment_lengths)
    f32 = torch.float32
    n0 = ctx.segment_lengths[0] if nseg else 0
    linear = None
    if SHARED_PREP and first_cont and fused_supported(q, v) and n0 >= 64:
        o, S_zero, L_rows, M_first = fused_affine_delta_rule(q, k, v, g, beta, layout,
                                                             _first_layout(ctx, layout, nseg, n0))
        linear = (L_rows, M_first[None])
    else:
        if first_cont:
            linear = _identity_pass(q, k, g, beta, n0, _first_layout(ctx, layout, nseg, n0))
        o, S_zero = _rule(q, k, v, g, beta, layout)
        if linear is not None and q.is_cuda:
            torch.cuda.current_stream(q.device).wait_stream(_side_stream(q.device))
            for t in linear:
                t.record_stream(torch.cuda.current_stream(q.device))
    F_tail = S_zero[nseg - 1] if last_cont else torch.zeros((H, DK, DV), dtype=f32, device=q.device)
    if last_cont and first_cont and single:
        M_tail = linear[1][0]
    else:
        M_tail = torch.zeros((H, DK, DK), dtype=f32, device=q.device)
    packed = torch.cat([F_tail.reshape(-1), M_tail.reshape(-1)])
    if torch.is_grad_enabled() and not packed.requires_grad:
        # a rank whose contribution is a constant must still own an all-gather
        # backward node, or the team's backward collectives would not match
        packed = packed.detach().requires_grad_(True)
    gathered = all_gather_rows(packed, ctx.team)
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
        # o_t += L_t S_in for the first segment's rows (one [n0, dk] x [dk, dv] product per head)
        corr = torch.einsum("thk,hkv->thv", linear[0].to(f32), state)
        o = torch.cat([(o[:n0].to(f32) + corr).to(o.dtype), o[n0:]], 0)
    return tie(o, gathered)
