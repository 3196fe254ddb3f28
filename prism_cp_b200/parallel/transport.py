"""CP-transition reshard: exact token permutation between two ownership layouts.

``move(x, source, target)`` moves this rank's rows of ``x`` (local order of
``source``) to their owners in ``target`` using the interval route of the IR;
the backward runs the inverse route (reference behaviour:
experiments/sequence_dynamic_cp/joint_cp/transport.py:12-70). Identity routes
(same rank, same offset) cost nothing. Two transports:

* P2P (``use_p2p``; the trainer's default on GPUs): the sender stages its rows
  in a symmetric heap and one gather kernel pulls them over NVLink into the
  destination layout (``parallel/symm.py``);
* NCCL (CPU / gloo, or ``PRISM_RESHARD=nccl``): an all-to-all with per-peer
  split sizes over the world.

Routes are compiled once per (source, target, lengths) into per-peer row index
tensors, so the pack and unpack are single gathers/scatters on the device.
"""

from __future__ import annotations

from functools import lru_cache

import torch
import torch.distributed as dist

from ..planner.joint.ir import identity_route, route


class CompiledRoute:
    def __init__(self, edges, world: int, rank: int, device):
        out = sorted((e for e in edges if e[0] == rank), key=lambda e: (e[1], e[2], e[3]))
        inc = sorted((e for e in edges if e[1] == rank), key=lambda e: (e[0], e[2], e[3]))
        self.send_sizes = [sum(e[4] for e in out if e[1] == p) for p in range(world)]
        self.recv_sizes = [sum(e[4] for e in inc if e[0] == p) for p in range(world)]
        self.rows_in = sum(e[4] for e in out)
        self.rows_out = sum(e[4] for e in inc)
        send_idx, recv_idx = [], []
        for _, _, src_off, _, n in out:
            send_idx.extend(range(src_off, src_off + n))
        for _, _, _, dst_off, n in inc:
            recv_idx.extend(range(dst_off, dst_off + n))
        self.send_index = torch.tensor(send_idx, dtype=torch.int64, device=device)
        self.recv_index = torch.tensor(recv_idx, dtype=torch.int64, device=device)
        self.remote = any(e[0] != e[1] for e in edges)
        self.world, self.rank = world, rank
        self.edges = tuple(edges)


def _exchange(x: torch.Tensor, r: CompiledRoute, group) -> torch.Tensor:
    if x.shape[0] != r.rows_in:
        raise ValueError("tensor does not match the compiled route")
    send = x.index_select(0, r.send_index)
    received = x.new_empty((r.rows_out,) + tuple(x.shape[1:]))
    if r.remote:
        dist.all_to_all_single(received, send.contiguous(), r.recv_sizes, r.send_sizes, group=group)
    else:
        received.copy_(send)
    out = x.new_empty((r.rows_out,) + tuple(x.shape[1:]))
    out.index_copy_(0, r.recv_index, received)
    return out


class _Permute(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fwd, bwd, group):
        ctx.bwd, ctx.group = bwd, group
        return _exchange(x, fwd, group)

    @staticmethod
    def backward(ctx, g):
        return _exchange(g.contiguous(), ctx.bwd, ctx.group), None, None, None


class _PermuteP2P(torch.autograd.Function):
    """The same permutation over NVLink P2P loads from the symmetric heap."""

    @staticmethod
    def forward(ctx, x, edges, inverse, p2p):
        ctx.inverse, ctx.p2p = inverse, p2p
        return p2p.exchange(x.contiguous(), edges)

    @staticmethod
    def backward(ctx, g):
        return ctx.p2p.exchange(g.contiguous(), ctx.inverse), None, None, None


_P2P = {"transport": None}


def use_p2p(transport) -> None:
    """Route every remote reshard through ``transport`` (a ``symm.P2PTransport``); None restores NCCL."""
    _P2P["transport"] = transport


@lru_cache(maxsize=512)
def _compiled(source, target, lengths_key, world, rank, device_str):
    lengths = dict(lengths_key)
    edges = route(source, target, lengths, world)
    if identity_route(edges):
        return None
    inverse = tuple((d, s, b, a, n) for s, d, a, b, n in edges)
    dev = torch.device(device_str)
    return CompiledRoute(edges, world, rank, dev), CompiledRoute(inverse, world, rank, dev)


def move(x: torch.Tensor, source, target, group=None) -> torch.Tensor:
    """Reshard rows of ``x`` from LocalLayout ``source`` to LocalLayout ``target``."""
    if source.layout == target.layout:
        return x
    if group is None:
        group = getattr(source, "world_group", None)
    lengths_key = tuple(sorted(source.lengths.items()))
    compiled = _compiled(source.layout, target.layout, lengths_key, source.world, source.rank, str(x.device))
    if compiled is None:
        return x
    fwd, bwd = compiled
    if _P2P["transport"] is not None and fwd.remote:
        return _PermuteP2P.apply(x, fwd.edges, bwd.edges, _P2P["transport"])
    return _Permute.apply(x, fwd, bwd, group)
