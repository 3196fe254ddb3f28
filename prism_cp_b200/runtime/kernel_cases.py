"""Small, self-contained kernel workloads for profilers (``ncu``) and quick timing.

``python -m prism_cp_b200.runtime.kernel_cases <case> [--iters N]`` runs one
case a few times on ``cuda:0`` and prints the CUDA-event time of the last
iteration. Every case keeps a few GB on the device at most, so an ``ncu``
capture of one of its kernels (``-k <kernel> -c 1``) ends in a minute or two.

Cases
  gdn        fused chunked gated delta rule fwd + bwd, 4 x 4096 tokens, 16 heads, dk 128, dv 256
  gdn32k     the same on one 32768-token sequence (one GDN layer of the 1.3B model at CP = 1)
  attention  causal GQA flash attention fwd + bwd, 2 x 8192 tokens, 16 query / 4 kv heads, d 128
  gemm       bf16 GEMM 16384 x 2048 x 8192 (forward projection shape of the 1.3B model)
  conv       causal conv1d + SiLU fwd + bwd, 32768 tokens x 8192 channels
"""

from __future__ import annotations

import argparse
import sys

import torch
import torch.nn.functional as F


def case_gdn(dev, lens=(4096,) * 4):
    from ..ops.gdn import ChunkLayout, fused_gated_delta_rule
    T, H = sum(lens), 16
    g = torch.Generator(device=dev).manual_seed(0)
    q = F.normalize(torch.randn(T, H, 128, device=dev, generator=g), dim=-1).to(torch.bfloat16).requires_grad_(True)
    k = F.normalize(torch.randn(T, H, 128, device=dev, generator=g), dim=-1).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(T, H, 256, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    gl = (-torch.rand(T, H, device=dev, generator=g) * 0.3).requires_grad_(True)
    beta = torch.rand(T, H, device=dev, generator=g).requires_grad_(True)
    layout = ChunkLayout(lens, dev)

    def run():
        o, _ = fused_gated_delta_rule(q, k, v, gl, beta, layout)
        o.float().sum().backward()
    return run


def case_attention(dev):
    from ..ops.attention import AttentionMeta, flash_attention
    lens = (8192, 8192)
    T = sum(lens)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(T, 16, 128, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(T, 4, 128, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(T, 4, 128, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    meta = AttentionMeta(lens, lens, True, dev)

    def run():
        o, _ = flash_attention(q, k, v, meta)
        o.float().sum().backward()
    return run


def case_gemm(dev):
    from ..ops.gemm import matmul
    a = torch.randn(16384, 2048, device=dev).to(torch.bfloat16)
    b = torch.randn(8192, 2048, device=dev).to(torch.bfloat16)

    def run():
        matmul(a, b)
    return run


def case_conv(dev):
    from ..ops.elementwise import causal_conv1d_silu
    x = torch.randn(32768, 8192, device=dev).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(8192, 4, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
    cu = torch.tensor([0, 16384, 32768], dtype=torch.int32, device=dev)

    def run():
        y = causal_conv1d_silu(x, w, cu)
        y.float().sum().backward()
    return run


def case_gdn32k(dev):
    return case_gdn(dev, (32768,))


CASES = {"gdn": case_gdn, "gdn32k": case_gdn32k, "attention": case_attention, "gemm": case_gemm, "conv": case_conv}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--no-sync", action="store_true", help="queue iterations back to back (host runs ahead)")
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    run = CASES[args.case](dev)
    from ..utils import watchdog
    watchdog.from_env()
    ms = 0.0
    for i in range(args.iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        watchdog.beat(f"iteration {i} queued")
        if not args.no_sync:
            torch.cuda.synchronize()
            ms = a.elapsed_time(b)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    from ..ops._lib import check_status
    check_status(dev)
    print(f"{args.case}: {ms:.3f} ms (last of {args.iters})")
    return 0


if __name__ == "__main__":
    sys.exit(main())
