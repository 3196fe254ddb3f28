"""Timing of the CP-transition reshard: NCCL all-to-all against the P2P gather over NVLink.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m prism_cp_b200.runtime.reshard_bench \\
        --seqs 8 --seq-len 32768 --hidden 2048

The workload is the GDN -> GQA boundary of the 1.3B benchmark at CP = N: ``seqs``
documents of ``seq-len`` tokens owned by one team of all N ranks, moved from the
contiguous layout (GDN) to the zigzag layout (GQA); rows are ``hidden`` bf16 values.
Two transports of ``parallel.transport.move`` are timed with CUDA events on the
launching stream after warm-up, max over ranks:

* ``nccl``: index-select of the outgoing rows, ``all_to_all_single``, index-copy
  into the destination layout (the default);
* ``p2p``: outgoing rows staged in the rank's symmetric heap, a bounded ready
  signal, then one gather kernel pulling every incoming row block from its
  owner's heap over NVLink straight into the destination layout.

The roofline is the bytes the busiest rank receives from other ranks at the
measured 770 GB/s peer-copy bandwidth per direction. One JSON line per run.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy per direction


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)

    from ..parallel import transport
    from ..parallel.layout import LocalLayout
    from ..parallel.symm import P2PTransport, SymmetricHeap
    from ..parallel.teams import Teams
    from ..planner.joint.ir import Group, Layout, route

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    world, rank = dist.get_world_size(), dist.get_rank()
    teams = Teams(world)
    lengths = {i: args.seq_len for i in range(args.seqs)}
    group = (Group(tuple(range(world)), tuple(range(args.seqs))),)
    src = LocalLayout(Layout(group, "contiguous"), lengths, world, rank, dev, teams)
    dst = LocalLayout(Layout(group, "zigzag"), lengths, world, rank, dev, teams)
    x = torch.randn(src.tokens, args.hidden, device=dev).to(torch.bfloat16)

    # bytes the busiest rank receives from other ranks
    edges = route(src.layout, dst.layout, lengths, world)
    incoming = [0] * world
    for s, d, _, _, n in edges:
        if s != d:
            incoming[d] += n * args.hidden * 2
    remote = max(incoming)

    ref = transport.move(x, src, dst)
    nccl_ms = _time(lambda: transport.move(x, src, dst), args.iters, args.warmup)
    heap = SymmetricHeap(teams.world_group, 4 * x.numel() * x.element_size() + (64 << 20), dev)
    transport.use_p2p(P2PTransport(heap))
    try:
        out = transport.move(x, src, dst)
        exact = bool(torch.equal(out, ref))
        p2p_ms = _time(lambda: transport.move(x, src, dst), args.iters, args.warmup)
    finally:
        transport.use_p2p(None)
    from ..ops._lib import check_status
    check_status(dev)
    roof_ms = remote / (LINK_GBS * 1e6)
    if rank == 0:
        print(json.dumps({"op": "cp_transition_reshard", "world": world, "seqs": args.seqs, "seq_len": args.seq_len,
                          "hidden": args.hidden, "rows_per_rank": src.tokens, "remote_bytes_max_rank": remote,
                          "nccl_ms": round(nccl_ms, 4), "p2p_ms": round(p2p_ms, 4), "p2p_equals_nccl": exact,
                          "roofline_ms": round(roof_ms, 4),
                          "nccl_fraction_of_roofline": round(roof_ms / nccl_ms, 3),
                          "p2p_fraction_of_roofline": round(roof_ms / p2p_ms, 3)}), flush=True)
    dist.barrier()
    heap.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
