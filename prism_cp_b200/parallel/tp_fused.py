"""Tensor-parallel GEMM fused with its all-reduce over NVLink peer memory.

``FusedAllReduceGemm(group)(a, b)`` returns ``sum over the TP ranks of a_r b_r^T``
(bf16) computed by one tcgen05 kernel per rank (``csrc/gemm_sm100.cu``, AR
mode): the tile rows are cut into one owner block per rank, each rank stores
its bf16 partials of the other owners' tiles straight into their staging slots
while its tensor cores continue with the next tiles, and every owner adds the
staged partials to its own fp32 accumulator and writes the finished tile into
every rank's output region. NVLink carries what a reduce-scatter plus an
all-gather would; no NCCL kernel and no separate reduction pass run.

Regions live in one symmetric heap per TP group (``symm.SymmetricHeap``):

    [ part_flag  t x max_tiles u64 | res_flag  max_tiles u64 | staging  t x R*128 x N bf16 | output  M x N bf16 ]

Flags hold the sequence number of the call that wrote them, so they are never
reset. A region is rewritten in call s+1 only after every rank finished call s
(a rank's call s+1 stores reach an owner only after that rank copied all of
call s's sums, which the owner produced after reading all of call s's
partials), so one copy of each region suffices. All calls on a group are
issued on one CUDA stream per rank, in the same order on every rank (they are
the TP layers of the model, run in lockstep). The heap grows (collectively, at
the same call on every rank: the TP group shares M and N) when a call needs
more room.

Used by ``tensor.row_linear`` (forward) and ``tensor.column_linear``
(backward input gradient) when the operands are on CUDA and ``PRISM_TP_FUSED=1``;
by default those sums run as NCCL reduce-scatter + all-gather, which measured faster.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops._lib import lib, status
from .symm import SymmetricHeap

BM, BN = 128, 256
# Measured on two B200s (16384 x 4096 x 2048, row-parallel): 1.20 ms fused against 0.60 ms for the
# GEMM followed by NCCL reduce-scatter + all-gather (0.24 ms GEMM alone; roofline 0.17 ms). The
# per-thread 64-byte stores to peer memory and a system-scope fence per tile hold the epilogue back,
# so the tensor cores wait. Opt-in until the epilogue stages tiles for bulk peer stores.
ENABLED = os.environ.get("PRISM_TP_FUSED", "0") == "1"


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class FusedAllReduceGemm:
    def __init__(self, group, device: torch.device):
        self.group, self.device = group, device
        self.t = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.heap: SymmetricHeap | None = None
        self.max_tiles = 0
        self.data_bytes = 0
        self.seq = 0

    def _ensure(self, tiles: int, data_bytes: int) -> None:
        if self.heap is not None and tiles <= self.max_tiles and data_bytes <= self.data_bytes:
            return
        if self.heap is not None:
            # every rank reaches this call together; peers finish with the old heap before it goes
            torch.cuda.current_stream(self.device).synchronize()
            dist.barrier(group=self.group)
            self.heap.close()
        self.max_tiles = max(tiles, 2 * self.max_tiles, 1024)
        self.data_bytes = max(data_bytes, self.data_bytes + self.data_bytes // 2)
        self.heap = SymmetricHeap(self.group, self._flag_bytes() + self.data_bytes, self.device)

    def _flag_bytes(self) -> int:
        return _align((self.t + 1) * self.max_tiles * 8)

    def __call__(self, a: torch.Tensor, b: torch.Tensor, b_mn: bool = False) -> torch.Tensor:
        M = a.shape[0]
        N = b.shape[1] if b_mn else b.shape[0]
        tiles_m, tiles_n = -(-M // BM), -(-N // BN)
        R = -(-tiles_m // self.t)
        ld = N
        staging = _align(self.t * R * BM * ld * 2)
        output = _align(tiles_m * BM * ld * 2)
        self._ensure(tiles_m * tiles_n, staging + output)
        flags = self._flag_bytes()
        bases = self.heap.bases
        regions = torch.tensor([[base + flags for base in bases],
                                [base + flags + staging for base in bases],
                                [base for base in bases],
                                [base + self.t * self.max_tiles * 8 for base in bases]], dtype=torch.int64)
        self.seq += 1
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
        lib().gemm_allreduce(a, b, out, False, b_mn, regions, self.me, self.max_tiles, ld, self.seq,
                             status(a.device))
        return out

    def close(self) -> None:
        if self.heap is not None:
            self.heap.close()
            self.heap = None


_FUSED: dict = {}


def fused_for(group, device: torch.device) -> FusedAllReduceGemm:
    key = (id(group), device.index)
    f = _FUSED.get(key)
    if f is None:
        f = FusedAllReduceGemm(group, device)
        _FUSED[key] = f
    return f


def usable(x: torch.Tensor, n: int, group) -> bool:
    """Whether the fused kernel applies: CUDA bf16 operands, 16-byte output rows, a real group."""
    return (ENABLED and group is not None and x.is_cuda and x.dtype == torch.bfloat16 and n % 8 == 0
            and 2 <= dist.get_world_size(group) <= 8)
