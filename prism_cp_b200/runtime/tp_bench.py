"""Timing of the tensor-parallel GEMM + all-reduce: fused kernel vs GEMM + NCCL.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m prism_cp_b200.runtime.tp_bench \\
        --tokens 16384 --out-features 4096 --in-features 2048

Every rank holds a [M, K] bf16 shard of the activations and a [N, K] shard of the
weight (a row-parallel linear: the 7B hybrid's attention output projection at
TP=2 is M tokens x N=4096 x K=2048). Three variants are timed with CUDA events
on the launching stream after warm-up, max over ranks:

* ``gemm``: the local partial product alone (the compute floor);
* ``unfused``: partial product, then NCCL reduce-scatter + all-gather;
* ``fused``: the tcgen05 GEMM that exchanges partial and finished tiles over
  NVLink peer memory (``parallel.tp_fused``).

The roofline of the fused op is the slower of its FLOPs at the measured bf16
GEMM peak and the bytes one rank sends over NVLink ((t-1)/t of the output as
partials plus the same again as finished tiles) at the measured 770 GB/s
peer-copy bandwidth per direction. One JSON line per run.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

PEAK_TFLOPS = 1663.7      # cuBLAS bf16 8192^3 burst on this B200 type
LINK_GBS = 770.0          # measured peer copy per direction


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
    # (long names: torchrun would take --m / --n / --k for abbreviations of its own options)
    ap.add_argument("--tokens", dest="m", type=int, default=16384)
    ap.add_argument("--out-features", dest="n", type=int, default=4096)
    ap.add_argument("--in-features", dest="k", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    t, rank = dist.get_world_size(), dist.get_rank()
    from ..ops._lib import check_status
    from ..ops.gemm import matmul
    from ..parallel.tp_fused import FusedAllReduceGemm

    g = torch.Generator(device=dev).manual_seed(rank)
    a = torch.randn(args.m, args.k, device=dev, generator=g).to(torch.bfloat16)
    b = (torch.randn(args.n, args.k, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    fused = FusedAllReduceGemm(dist.group.WORLD, dev)

    def run_gemm():
        return matmul(a, b)

    def run_unfused():
        y = matmul(a, b)
        part = torch.empty((args.m // t, args.n), dtype=y.dtype, device=dev)
        dist.reduce_scatter_tensor(part, y)
        out = torch.empty_like(y)
        dist.all_gather_into_tensor(out, part)
        return out

    def run_fused():
        return fused(a, b)

    # numerics first: the fused result against the unfused one
    ref, got = run_unfused(), run_fused()
    torch.cuda.synchronize()
    check_status(dev)
    err = float(((got.float() - ref.float()).norm() / ref.float().norm()).item())
    ms_gemm = _time(run_gemm, args.iters, args.warmup)
    ms_unfused = _time(run_unfused, args.iters, args.warmup)
    ms_fused = _time(run_fused, args.iters, args.warmup)
    check_status(dev)
    flops = 2.0 * args.m * args.n * args.k
    link_bytes = 2.0 * (t - 1) / t * args.m * args.n * 2
    roof_ms = max(flops / (PEAK_TFLOPS * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e3
    if rank == 0:
        print(json.dumps({
            "op": "tp_gemm_allreduce", "tp": t, "m": args.m, "n": args.n, "k": args.k,
            "ms_gemm_only": round(ms_gemm, 4), "ms_unfused_nccl": round(ms_unfused, 4),
            "ms_fused": round(ms_fused, 4), "speedup_vs_unfused": round(ms_unfused / ms_fused, 3),
            "roofline_ms": round(roof_ms, 4), "fraction_of_roofline": round(roof_ms / ms_fused, 3),
            "fused_tflops": round(flops / ms_fused / 1e9, 1), "nvlink_bytes_per_rank": int(link_bytes),
            "rel_err_vs_unfused": err, "timing": "CUDA events, max over ranks",
            "l2": "operands + output exceed the 126 MB L2"}), flush=True)
    fused.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
