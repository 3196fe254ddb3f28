"""Symmetric heaps over NVLink and the P2P CP-transition reshard built on them.

``SymmetricHeap(group, nbytes)`` allocates ``nbytes`` (plus a signal region) on
every rank of ``group`` with ``cudaMalloc``, exchanges CUDA IPC handles over the
group once, and opens every peer's heap, so device code can load and store
peer memory directly. Signal slots are 64-bit sequence words written with
system-scope release stores and waited on with bounded acquire spins
(``csrc/symm.cu``): a peer that never arrives produces an error status, not a
hang.

``P2PTransport`` replaces the reshard's NCCL all-to-all (``transport.py``): each
rank stages its outgoing rows in its heap, publishes a ready signal, and one
gather kernel pulls every incoming row block straight from the owner's heap
into the destination layout (16-byte loads over NVLink). Staging alternates
between two halves of the heap by sequence parity, and a rank only rewrites
a half after every peer has signalled that it finished reading it.
"""

from __future__ import annotations

import math
import os

import torch
import torch.distributed as dist

from ..ops._lib import lib, status

SIGNAL_SLOTS = 256
READY, DONE = 0, 64      # slot bases: READY + src_rank, DONE + src_rank
# how long a signal wait tolerates a late peer before it records an error (bounded; a rank that is
# seconds behind its peers inside one step is a fault, not load imbalance)
PEER_WAIT_NS = int(float(os.environ.get("PRISM_PEER_WAIT_S", "20")) * 1e9)


class SymmetricHeap:
    def __init__(self, group, nbytes: int, device: torch.device, wait_ns: int | None = None):
        self.group = group
        self.wait_ns = PEER_WAIT_NS if wait_ns is None else int(wait_ns)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = (nbytes + 255) // 256 * 256
        self.device = device
        L = lib()
        total = self.nbytes + SIGNAL_SLOTS * 8
        self.local = L.symm_alloc(total)
        handle = L.symm_handle(self.local)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.numpy().tobytes(), group=group)
        self.bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.local)
            else:
                self.bases.append(L.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
        self.bases_dev = torch.tensor(self.bases, dtype=torch.int64, device=device)
        self.signal_dev = self.bases_dev + self.nbytes
        self.my_signals = self.local + self.nbytes
        self.seq = 0

    def view(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        code = {torch.bfloat16: 15, torch.float32: 6, torch.int64: 4, torch.uint8: 0, torch.float16: 5}[dtype]
        return lib().symm_tensor(self.local + offset, list(shape), code, self.device.index)

    def signal(self, slot: int, value: int):
        lib().symm_signal(self.signal_dev, slot, value)

    def wait(self, first: int, count: int, value: int):
        lib().symm_wait(self.my_signals, first, count, value, status(self.device), self.wait_ns)

    def close(self):
        L = lib()
        for r, b in enumerate(self.bases):
            if r != self.rank:
                L.symm_close(b)
        L.symm_free(self.local)


class _CompiledP2PRoute:
    def __init__(self, edges, rank: int, row_bytes: int, rows_per_block: int, device, send_rows_by_rank):
        # the sender stages its outgoing rows in source-offset order; offsets of
        # each sender's rows inside its staging area are known to every rank
        routes, block_route, block_row0 = [], [], []
        incoming = sorted((e for e in edges if e[1] == rank), key=lambda e: (e[0], e[2]))
        for s, _, src_off, dst_off, n in incoming:
            staged = send_rows_by_rank[s][(src_off, n)]
            routes.append((s, staged * row_bytes, dst_off * row_bytes, n))
            for r0 in range(0, n, rows_per_block):
                block_route.append(len(routes) - 1)
                block_row0.append(r0)
        self.routes = torch.tensor(routes or [(0, 0, 0, 0)], dtype=torch.int64, device=device)
        self.block_route = torch.tensor(block_route, dtype=torch.int64, device=device)
        self.block_row0 = torch.tensor(block_row0, dtype=torch.int64, device=device)
        out = sorted((e for e in edges if e[0] == rank), key=lambda e: e[2])
        idx = [torch.arange(src_off, src_off + n, dtype=torch.int64) for _, _, src_off, _, n in out]
        self.send_index = (torch.cat(idx) if idx else torch.zeros(0, dtype=torch.int64)).to(device)
        self.rows_out = sum(e[4] for e in incoming)
        self.row_bytes, self.rows_per_block = row_bytes, rows_per_block


def staging_offsets(edges, world: int):
    """Per sender: (src_off, count) -> row index inside its staging area."""
    table = [dict() for _ in range(world)]
    for s in range(world):
        pos = 0
        for _, _, src_off, _, n in sorted((e for e in edges if e[0] == s), key=lambda e: e[2]):
            table[s][(src_off, n)] = pos
            pos += n
    return table


class P2PTransport:
    """Reshard rows between two layouts with P2P loads over NVLink (no NCCL).

    The staging heap is allocated on first use and regrown (after a barrier of the group) when a
    route needs more than half of it; the size comes from the global route (the largest number of
    rows any rank sends), so every rank makes the same decision at the same call."""

    def __init__(self, heap: SymmetricHeap | None = None, rows_per_block: int = 64, group=None,
                 device: torch.device | None = None, min_bytes: int = 256 << 20):
        self.heap = heap
        self.group = heap.group if heap is not None else group
        self.device = heap.device if heap is not None else device
        self.rows_per_block = rows_per_block
        self.min_bytes = min_bytes
        self.half = heap.nbytes // 2 if heap is not None else 0
        self._routes: dict = {}  # (edges, row bytes) -> compiled block tables, built once per route

    def _ensure(self, need: int) -> SymmetricHeap:
        if self.heap is None or need > self.half:
            if self.heap is not None:
                dist.barrier(group=self.group)
                self.heap.close()
            self.heap = SymmetricHeap(self.group, max(2 * need, self.min_bytes), self.device)
            self.half = self.heap.nbytes // 2
        return self.heap

    def close(self):
        if self.heap is not None:
            self.heap.close()
            self.heap = None

    def exchange(self, x: torch.Tensor, edges) -> torch.Tensor:
        # from the row shape, not from a local row: a rank's local part may be empty, and the route's
        # staging size (hence the heap decision) must be the same number on every rank
        row_bytes = math.prod(x.shape[1:]) * x.element_size()
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        key = (edges, row_bytes)
        r = self._routes.get(key)
        if r is None:
            r = _CompiledP2PRoute(edges, rank, row_bytes, self.rows_per_block, x.device,
                                  staging_offsets(edges, world))
            sent = [0] * world
            for s_, _, _, _, n in edges:
                sent[s_] += n
            r.max_stage_bytes = max(1, max(sent)) * row_bytes
            if len(self._routes) >= 512:
                self._routes.clear()
            self._routes[key] = r
        heap = self._ensure(r.max_stage_bytes)
        heap.seq += 1
        seq = heap.seq
        parity = seq % 2
        if seq > 2:
            # every peer has finished reading this half (from step seq - 2)
            heap.wait(DONE, heap.world, seq - 2)
        stage = heap.view(parity * self.half, (r.send_index.numel(),) + tuple(x.shape[1:]), x.dtype)
        if r.send_index.numel():
            torch.index_select(x, 0, r.send_index, out=stage)
        heap.signal(READY + heap.rank, seq)
        heap.wait(READY, heap.world, seq)
        out = x.new_empty((r.rows_out,) + tuple(x.shape[1:]))
        bases = heap.bases_dev + parity * self.half
        lib().symm_gather_rows(bases, r.routes, r.block_route, r.block_row0, r.rows_per_block, row_bytes, out,
                               status(x.device))
        heap.signal(DONE + heap.rank, seq)
        return out
