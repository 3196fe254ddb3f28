"""Zigzag context-parallel attention whose kernels read peer tiles over NVLink.

Instead of rotating K/V around a ring with NCCL and merging partial outputs,
every rank of the team places the tensors a kernel needs in a symmetric heap
(``symm.SymmetricHeap``) and the tcgen05 attention kernels load each tile from
the rank that owns it (``csrc/attention_peer.cuh``):

* forward: this rank's query tiles over the team's keys - K/V tiles are TMA
  loads from the owner's heap, so the exchange overlaps the tile loop and the
  output needs no LSE merge;
* backward: dK/dV for this rank's key tiles iterate over the team's query tiles
  (Q/dO from the owner, LSE/D rows read over NVLink), dQ for this rank's query
  tiles iterates over the team's K/V. Both are atomic-free.

Per call the heap region alternates between two halves; a rank overwrites a half
only after every peer has signalled that it finished reading it (bounded signal
waits, ``csrc/symm.cu``). Requirements: causal attention, every sequence length a
multiple of 256 * cp (chunks of whole 128-token tiles); other layouts use the
NCCL ring (``cp_attention.ZigzagRing``). Same semantics as the reference's CP
attention (TransformerEngine p2p ring, external to the reference).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._lib import lib, status
from .symm import SymmetricHeap

READY, DONE = 0, 64
_HEAPS: dict = {}


def _align(n: int) -> int:
    return (n + 255) // 256 * 256


def supported(ctx) -> bool:
    """Whether every sequence of this layout splits into whole 128-token chunks."""
    if ctx.cp < 2 or ctx.cp > 8 or ctx.mode != "zigzag":
        return False
    return all(ctx.lengths[s] % (256 * ctx.cp) == 0 for s in ctx.samples)


class TeamHeap:
    """A symmetric heap per team with a call sequence for the two-half protocol."""

    def __init__(self, ctx, nbytes: int):
        self.heap = SymmetricHeap(ctx.team, nbytes, ctx.device)
        self.ranks = ctx.group_ranks
        self.index = ctx.index
        self.seq = 0
        self.half = self.heap.nbytes // 2

    def begin(self, need: int) -> int:
        if need > self.half:
            raise ValueError(f"attention needs {need} heap bytes per call, half of the heap is {self.half}")
        self.seq += 1
        if self.seq > 2:
            self.heap.wait(DONE, len(self.ranks), self.seq - 2)
        return (self.seq % 2) * self.half

    def ready(self):
        self.heap.signal(READY + self.index, self.seq)
        self.heap.wait(READY, len(self.ranks), self.seq)

    def done(self):
        self.heap.signal(DONE + self.index, self.seq)

    def local(self, offset: int, shape, dtype) -> torch.Tensor:
        return self.heap.view(offset, shape, dtype)

    def peers(self, offset: int, shape, dtype) -> list[torch.Tensor]:
        code = {torch.bfloat16: 15, torch.float32: 6}[dtype]
        dev = self.heap.device.index
        return [lib().symm_tensor(base + offset, list(shape), code, dev) for base in self.heap.bases]


def team_heap(ctx, need: int) -> TeamHeap:
    key = ctx.group_ranks
    h = _HEAPS.get(key)
    if h is None or h.half < need:
        # every rank of the team reaches this point in the same call (layers run in lockstep)
        if h is not None:
            dist.barrier(group=ctx.team)
            h.heap.close()
        h = TeamHeap(ctx, max(2 * need, 64 << 20))
        _HEAPS[key] = h
    return h


class PeerAttention:
    def __init__(self, ctx):
        self.ctx = ctx
        dev = ctx.device
        seq_n, seq_row0, tiles = [], [], []
        cp, r = ctx.cp, ctx.index
        for s_idx, s in enumerate(ctx.samples):
            own = [sp for sp in ctx.spans if sp[0] == s]
            n = ctx.lengths[s]
            c = n // (2 * cp)
            row0 = min(sp[2] for sp in own)
            seq_n.append(n)
            seq_row0.append(row0)
            for begin, local in ((r * c, row0), ((2 * cp - 1 - r) * c, row0 + c)):
                for t in range(0, c, 128):
                    tiles.append((s_idx, begin + t, local + t))
        tiles.sort(key=lambda x: -x[1])  # longest causal rows first
        self.tiles = torch.tensor(tiles, dtype=torch.int32, device=dev).reshape(-1, 3)
        self.seq_n = torch.tensor(seq_n, dtype=torch.int32, device=dev)
        self.seq_row0 = torch.tensor(seq_row0, dtype=torch.int32, device=dev)

    def __call__(self, q, k, v, scale=None):
        scale = q.shape[-1] ** -0.5 if scale is None else scale
        return _PeerAttnFn.apply(q, k, v, self, scale)

    # ---------------------------------------------------------------- forward
    def forward(self, q, k, v, scale):
        T, Hq, D = q.shape
        Hkv = k.shape[1]
        kv_bytes = _align(T * Hkv * D * 2)
        heap = team_heap(self.ctx, 2 * kv_bytes)
        base = heap.begin(2 * kv_bytes)
        heap.local(base, (T, Hkv, D), torch.bfloat16).copy_(k)
        heap.local(base + kv_bytes, (T, Hkv, D), torch.bfloat16).copy_(v)
        heap.ready()
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=q.device)
        lse = torch.empty((Hq, T), dtype=torch.float32, device=q.device)
        lib().attention_fwd_peer(q.contiguous(), heap.peers(base, (T, Hkv, D), torch.bfloat16),
                                 heap.peers(base + kv_bytes, (T, Hkv, D), torch.bfloat16), self.tiles, self.seq_n,
                                 self.seq_row0, out, lse, scale, status(q.device))
        heap.done()
        return out, lse

    # ---------------------------------------------------------------- backward
    def backward(self, q, k, v, out, lse, dout, scale):
        T, Hq, D = q.shape
        Hkv = k.shape[1]
        bf, f32 = torch.bfloat16, torch.float32
        sizes = [("q", (T, Hq, D), bf), ("k", (T, Hkv, D), bf), ("v", (T, Hkv, D), bf), ("do", (T, Hq, D), bf),
                 ("lse", (Hq, T), f32), ("dsum", (Hq, T), f32)]
        offs, total = {}, 0
        for name, shape, dt in sizes:
            offs[name] = total
            n = 1
            for x in shape:
                n *= x
            total += _align(n * (2 if dt == bf else 4))
        heap = team_heap(self.ctx, total)
        base = heap.begin(total)
        views = {name: heap.local(base + offs[name], shape, dt) for name, shape, dt in sizes}
        views["q"].copy_(q)
        views["k"].copy_(k)
        views["v"].copy_(v)
        views["do"].copy_(dout)
        views["lse"].copy_(lse)
        lib().attention_bwd_dsum(out, views["do"], views["dsum"])
        heap.ready()
        peers = {name: heap.peers(base + offs[name], shape, dt) for name, shape, dt in sizes}
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        lib().attention_bwd_peer(peers["q"], peers["k"], peers["v"], peers["do"], peers["lse"], peers["dsum"],
                                 self.ctx.index, self.tiles, self.seq_n, self.seq_row0, dq, dk, dv, scale,
                                 status(q.device))
        heap.done()
        return dq, dk, dv


class _PeerAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, attn, scale):
        qb, kb, vb = (t.to(torch.bfloat16).contiguous() for t in (q, k, v))
        out, lse = attn.forward(qb, kb, vb, scale)
        ctx.save_for_backward(qb, kb, vb, out, lse)
        ctx.attn, ctx.scale = attn, scale
        ctx.dtypes = (q.dtype, k.dtype, v.dtype)
        return out.to(q.dtype)

    @staticmethod
    def backward(ctx, dout):
        qb, kb, vb, out, lse = ctx.saved_tensors
        dq, dk, dv = ctx.attn.backward(qb, kb, vb, out, lse, dout.to(torch.bfloat16).contiguous(), ctx.scale)
        tq, tk, tv = ctx.dtypes
        return dq.to(tq), dk.to(tk), dv.to(tv), None, None
