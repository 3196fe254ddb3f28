"""Module bench: one GQA, GDN or MLP block of the hybrid model, timed at CP = world.

Run on one GPU (``python -m prism_cp_b200.runtime.module_bench ...``) for CP 1,
or under ``torch.distributed.run --nproc-per-node p`` for CP p (one team of all
ranks: contiguous layout for GDN, zigzag for GQA). Before timing, the P0 gates
of the reference bench run (experiments/performance_model/module_bench.py):

* ``repeat``   - two runs on the same input give the same Y, dX and dW up to
  summation order (the GDN backward reduces per-chunk decay/beta terms with
  shared-memory atomics, so small parameters such as A_log can differ in the
  last bits; the bound is the reference's 5e-3);
* ``reference``- the module against an fp32 PyTorch evaluation of the same
  weights (attention / delta rule / MLP core on the CPU-reference code paths);
* ``packed``   - a packed batch of two sequences equals the two run separately.

Timing: ``warmup`` untimed iterations, then ``iterations`` timed forward,
backward and forward+backward passes with CUDA events on the launching
stream; each value is the max over ranks. Output: a JSON document with
``model_shape`` and ``records`` ({module, cp, tokens, sequences, f_ms, b_ms,
fb_ms}), the input of ``planner.profile_builder`` and ``planner.costfit``.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

THRESHOLDS = {"repeat": 5e-3, "reference": 3e-2, "packed": 1e-2}


def rel(a, b) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def build(module: str, cfg, device, seed: int):
    from ..models.hybrid import MLP, GDNMixer, GQAMixer
    gen = torch.Generator().manual_seed(seed)
    cls = {"gqa": GQAMixer, "gdn": GDNMixer, "mlp": MLP}[module]
    return cls(cfg, torch.bfloat16, device, gen)


def layout_for(module: str, lengths: dict, world: int, rank: int, device, teams):
    from ..parallel.layout import LocalLayout
    from ..planner.joint.ir import Group, Layout
    mode = "contiguous" if module == "gdn" else "zigzag"
    return LocalLayout(Layout((Group(tuple(range(world)), tuple(sorted(lengths))),), mode), lengths, world, rank,
                       device, teams)


def run_once(mod, module: str, x, ctx):
    x = x.detach().requires_grad_(True)
    for p in mod.parameters():
        p.grad = None
    y = mod(x) if module == "mlp" else mod(x, ctx)
    g = torch.ones_like(y) / y.numel() ** 0.5
    y.backward(g)
    grads = [p.grad.detach().clone() for p in mod.parameters() if p.grad is not None]
    return y.detach(), x.grad.detach(), grads


def local_rows(ctx, full: torch.Tensor, offsets: dict) -> torch.Tensor:
    idx = [offsets[s] + b + j for s, b, _, c in ctx.spans for j in range(c)]
    return full[torch.tensor(idx, device=full.device)]


def gates(mod, module, cfg, device, world, rank, teams) -> dict:
    """P0 numerical gates on a small case; raises if a gate fails."""
    lengths = {0: 1024 * world, 1: 512 * world}
    ctx = layout_for(module, lengths, world, rank, device, teams)
    g = torch.Generator(device=device).manual_seed(7)
    full = torch.randn(sum(lengths.values()), cfg.hidden_size, device=device, generator=g).to(torch.bfloat16)
    x = local_rows(ctx, full, {0: 0, 1: lengths[0]})
    y1, dx1, w1 = run_once(mod, module, x, ctx)
    y2, dx2, w2 = run_once(mod, module, x, ctx)
    out = {"repeat": max(rel(y2, y1), rel(dx2, dx1), max(rel(a, b) for a, b in zip(w2, w1)))}
    if world == 1:
        # packed vs separate
        sep = []
        for s, n in lengths.items():
            c1 = layout_for(module, {0: n}, 1, 0, device, teams)
            start = 0 if s == 0 else lengths[0]
            sep.append(run_once(mod, module, full[start:start + n], c1)[0])
        out["packed"] = rel(y1, torch.cat(sep))
        # fp32 reference core: same weights in fp32 on the CPU reference paths
        ref_mod = build(module, cfg, torch.device("cpu"), 0)
        ref_mod.load_state_dict({k: v.detach().float().cpu() for k, v in mod.state_dict().items()})
        ref_mod = ref_mod.float()
        from ..parallel.layout import LocalLayout, single_rank_layout
        cpu_ctx = LocalLayout(single_rank_layout(lengths, "contiguous" if module == "gdn" else "zigzag"), lengths,
                              1, 0, torch.device("cpu"))
        yr = ref_mod(x.float().cpu()) if module == "mlp" else ref_mod(x.float().cpu(), cpu_ctx)
        out["reference"] = rel(y1.float().cpu(), yr)
    for k, v in out.items():
        if not v <= THRESHOLDS[k]:
            raise RuntimeError(f"P0 gate {k} failed for {module}: {v:.3g} > {THRESHOLDS[k]}")
    return out


def time_case(mod, module, cfg, device, world, rank, teams, seq_lens, warmup, iterations) -> dict:
    lengths = dict(enumerate(seq_lens))
    ctx = layout_for(module, lengths, world, rank, device, teams)
    x = torch.randn(ctx.tokens, cfg.hidden_size, device=device).to(torch.bfloat16)
    stream = torch.cuda.current_stream()

    def fwd():
        xi = x.detach().requires_grad_(True)
        return xi, (mod(xi) if module == "mlp" else mod(xi, ctx))

    for _ in range(warmup):
        _, y = fwd()
        y.backward(torch.ones_like(y))
    torch.cuda.synchronize()
    f_ms, b_ms = [], []
    for _ in range(iterations):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record(stream)
        _, y = fwd()
        e[1].record(stream)
        y.backward(torch.ones_like(y))
        e[2].record(stream)
        torch.cuda.synchronize()
        f_ms.append(e[0].elapsed_time(e[1]))
        b_ms.append(e[1].elapsed_time(e[2]))
    vals = torch.tensor([sorted(f_ms)[len(f_ms) // 2], sorted(b_ms)[len(b_ms) // 2]], dtype=torch.float64,
                        device=device)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    f, b = vals.tolist()
    return {"module": {"gqa": "GQA", "gdn": "GDN", "mlp": "M"}[module], "cp": world, "tokens": sum(seq_lens),
            "sequences": len(seq_lens), "f_ms": f, "b_ms": b, "fb_ms": f + b}


def parse_case(text: str) -> list[int]:
    """'32768' -> one sequence; '4x8192' -> four sequences of 8192 tokens."""
    if "x" in text:
        n, length = text.split("x")
        return [int(length)] * int(n)
    return [int(text)]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--module", choices=("gqa", "gdn", "mlp"), required=True)
    ap.add_argument("--model", default="hybrid-1.3b")
    ap.add_argument("--cases", default="8192,16384,32768,65536,4x8192")
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iterations", type=int, default=10)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--skip-gates", action="store_true")
    args = ap.parse_args(argv)
    from ..models.config import PRESETS
    from ..parallel.teams import Teams
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    cfg = PRESETS[args.model]()
    teams = Teams(world)
    mod = build(args.module, cfg, device, args.seed)
    t0 = time.perf_counter()
    gate = {} if args.skip_gates else gates(mod, args.module, cfg, device, world, rank, teams)
    records = []
    for case in args.cases.split(","):
        seq = parse_case(case)
        if any(n % (2 * world) for n in seq):
            continue
        records.append(time_case(mod, args.module, cfg, device, world, rank, teams, seq, args.warmup,
                                 args.iterations))
        if rank == 0:
            print(json.dumps(records[-1]), flush=True)
    if rank == 0:
        shape = (cfg.hidden_size, cfg.num_attention_heads, cfg.num_query_groups, cfg.kv_channels,
                 cfg.linear_num_key_heads, cfg.linear_key_head_dim)
        doc = {"model": cfg.name, "model_shape": list(shape), "world": world, "gates": gate, "records": records,
               "timing": "CUDA events on the launching stream, median of iterations, max over ranks",
               "wall_seconds": time.perf_counter() - t0, "device": torch.cuda.get_device_name(device)}
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(doc, indent=2) + "\n")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
