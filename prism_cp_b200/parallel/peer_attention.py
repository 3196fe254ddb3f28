"""Zigzag context-parallel attention over a symmetric heap (no ring, no LSE merge).

Every rank of the team stages the tensors the attention kernels need in a
symmetric heap (``symm.SymmetricHeap``); after a bounded ready signal each rank
pulls the peers' slabs into local memory with one P2P gather kernel (16-byte
loads over NVLink, every byte crosses NVLink once; its own slab is read in
place), and the tcgen05 attention
kernels then run over the whole sequence in global positions
(``csrc/attention_peer.cuh``), reading the slab of the rank that owns each tile:

* forward: this rank's query tiles over the team's keys (K/V slabs);
* backward: dK/dV for this rank's key tiles over the team's query tiles (Q/dO
  slabs and their LSE / D rows), dQ for this rank's query tiles over the team's
  K/V. Both are atomic-free and need no partial-result exchange.

Reading peer tiles straight from the peers' heaps inside the tile loop re-reads
each remote K/V tile once per query tile over NVLink, which made the kernels
NVLink-bound; pulling the slabs once keeps NVLink traffic at the all-gather
volume and the tile loop on HBM. Per call the heap region alternates between two
halves; a rank overwrites a half only after every peer has signalled that it
finished reading it (bounded signal waits, ``csrc/symm.cu``). Requirements:
causal attention, every sequence length a multiple of 256 * cp; other layouts
use the NCCL ring (``cp_attention.ZigzagRing``). Same semantics as the
reference's CP attention (TransformerEngine p2p ring, external to the reference).
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
        self._gather_plans: dict = {}

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

    def gather(self, offset: int, shape, dtype, local: torch.Tensor | None = None,
               rows_per_block: int = 64) -> list[torch.Tensor]:
        """Every team rank's region [offset, offset + size) as a list of slabs in team order:
        the peers' regions copied into one local buffer by a single P2P gather launch, and this
        rank's own slab taken as ``local`` (no copy) when given."""
        n = len(self.ranks)
        rows = shape[0]
        row_bytes = torch.tensor([], dtype=dtype).element_size()
        for x in shape[1:]:
            row_bytes *= x
        sources = [r for r in range(n) if local is None or r != self.index]
        out = torch.empty((len(sources),) + tuple(shape), dtype=dtype, device=self.heap.device)
        key = (offset, tuple(shape), dtype, rows_per_block, local is None)
        plan = self._gather_plans.get(key)
        if plan is None:
            routes, block_route, block_row0 = [], [], []
            for slot, r in enumerate(sources):
                routes.append((r, offset, slot * rows * row_bytes, rows))
                for r0 in range(0, rows, rows_per_block):
                    block_route.append(slot)
                    block_row0.append(r0)
            dev = self.heap.device
            plan = (torch.tensor(routes, dtype=torch.int64, device=dev),
                    torch.tensor(block_route, dtype=torch.int64, device=dev),
                    torch.tensor(block_row0, dtype=torch.int64, device=dev))
            self._gather_plans[key] = plan
        if sources:
            lib().symm_gather_rows(self.heap.bases_dev, plan[0], plan[1], plan[2], rows_per_block, row_bytes, out,
                                   status(self.heap.device))
        slabs = list(out.unbind(0))
        if local is not None:
            slabs.insert(self.index, local)
        return slabs


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
        k_all = heap.gather(base, (T, Hkv, D), torch.bfloat16, local=k)
        v_all = heap.gather(base + kv_bytes, (T, Hkv, D), torch.bfloat16, local=v)
        heap.done()
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=q.device)
        lse = torch.empty((Hq, T), dtype=torch.float32, device=q.device)
        lib().attention_fwd_peer(q.contiguous(), k_all, v_all, self.tiles, self.seq_n, self.seq_row0, out, lse,
                                 scale, status(q.device))
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
        # this rank's own slabs are read in place from the heap (local memory); only peers' cross NVLink
        slabs = {name: heap.gather(base + offs[name], shape, dt, local=views[name]) for name, shape, dt in sizes}
        heap.done()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        lib().attention_bwd_peer(slabs["q"], slabs["k"], slabs["v"], slabs["do"], slabs["lse"], slabs["dsum"],
                                 self.ctx.index, self.tiles, self.seq_n, self.seq_row0, dq, dk, dv, scale,
                                 status(q.device))
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
