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

import torch
import torch.distributed as dist

from ..ops._lib import lib, status

SIGNAL_SLOTS = 256
READY, DONE = 0, 64      # slot bases: READY + src_rank, DONE + src_rank


class SymmetricHeap:
    def __init__(self, group, nbytes: int, device: torch.device):
        self.group = group
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
        lib().symm_wait(self.my_signals, first, count, value, status(self.device))

    def close(self):
        L = lib()
        for r, b in enumerate(self.bases):
            if r != self.rank:
                L.symm_close(b)
        L.symm_free(self.local)


class _CompiledP2PRoute:
    def __init__(self, edges, rank: int, row_bytes: int, rows_per_block: int, device, half_bytes: int,
                 send_rows_by_rank):
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
    """Reshard rows between two layouts with P2P loads over NVLink (no NCCL)."""

    def __init__(self, heap: SymmetricHeap, rows_per_block: int = 64):
        self.heap = heap
        self.rows_per_block = rows_per_block
        self.half = heap.nbytes // 2
        self._routes: dict = {}  # (edges, row bytes) -> compiled block tables, built once per route

    def exchange(self, x: torch.Tensor, edges) -> torch.Tensor:
        heap = self.heap
        row_bytes = x[0].numel() * x.element_size() if x.shape[0] else 0
        key = (edges, row_bytes)
        r = self._routes.get(key)
        if r is None:
            r = _CompiledP2PRoute(edges, heap.rank, row_bytes, self.rows_per_block, x.device, self.half,
                                  staging_offsets(edges, heap.world))
            if len(self._routes) >= 512:
                self._routes.clear()
            self._routes[key] = r
        need = max(1, r.send_index.numel()) * row_bytes
        if need > self.half:
            raise ValueError(f"reshard needs {need} staging bytes, heap half is {self.half}")
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
