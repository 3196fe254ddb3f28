"""Multi-GPU checks, run as ``torchrun --nproc-per-node N tests/mgpu_worker.py`` by test_multigpu.py.

Every rank compares the distributed result of its rows with the same op computed
on its own GPU over the whole problem (deterministic inputs, same seed).
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from prism_cp_b200.ops._lib import check_status  # noqa: E402
from prism_cp_b200.ops.attention import AttentionMeta, flash_attention  # noqa: E402
from prism_cp_b200.ops.gdn import ChunkLayout, chunk_gated_delta_rule  # noqa: E402
from prism_cp_b200.parallel.layout import LocalLayout  # noqa: E402
from prism_cp_b200.parallel.symm import P2PTransport, SymmetricHeap  # noqa: E402
from prism_cp_b200.parallel.teams import Teams  # noqa: E402
from prism_cp_b200.parallel.transport import move, use_p2p  # noqa: E402
from prism_cp_b200.planner.joint.ir import Group, Layout  # noqa: E402


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def rows_of(ctx, offsets):
    return torch.tensor([offsets[s] + b + j for s, b, _, c in ctx.spans for j in range(c)], device="cuda")


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    world, rank = dist.get_world_size(), dist.get_rank()
    teams = Teams(world)
    ranks = tuple(range(world))

    # 1. P2P reshard == NCCL reshard (forward and inverse backward)
    lengths = {0: 512 * world, 1: 256 * world, 2: 128 * world}
    a = LocalLayout(Layout((Group(ranks, (0, 1, 2)),), "zigzag"), lengths, world, rank, dev, teams)
    b = LocalLayout(Layout((Group(ranks, (0, 1, 2)),), "contiguous"), lengths, world, rank, dev, teams)
    torch.manual_seed(rank)
    x = torch.randn(a.tokens, 2048, device=dev, dtype=torch.bfloat16, requires_grad=True)
    y_nccl = move(x, a, b)
    (y_nccl.float() * 2).sum().backward()
    g_nccl = x.grad.clone()
    x.grad = None
    heap = SymmetricHeap(dist.group.WORLD, 256 << 20, dev)
    use_p2p(P2PTransport(heap))
    y_p2p = move(x, a, b)
    (y_p2p.float() * 2).sum().backward()
    use_p2p(None)
    torch.cuda.synchronize()
    check_status(dev)
    assert torch.equal(y_p2p, y_nccl), "P2P reshard differs from NCCL"
    assert torch.equal(x.grad, g_nccl), "P2P inverse reshard differs from NCCL"

    # 2. zigzag ring attention on the tcgen05 kernels vs one-GPU attention
    alen = {0: 4096, 1: 2048}
    ctx = LocalLayout(Layout((Group(ranks, (0, 1)),), "zigzag"), alen, world, rank, dev, teams)
    g = torch.Generator(device="cuda").manual_seed(11)
    T, Hq, Hkv, d = 6144, 8, 2, 128
    q = torch.randn(T, Hq, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(T, Hkv, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(T, Hkv, d, device=dev, generator=g).to(torch.bfloat16)
    go = torch.randn(T, Hq, d, device=dev, generator=g).to(torch.bfloat16)
    qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
    full, _ = flash_attention(qf, kf, vf, AttentionMeta((4096, 2048), (4096, 2048), True, dev))
    (full.float() * go.float()).sum().backward()
    rows = rows_of(ctx, {0: 0, 1: 4096})
    ql, kl, vl = (t[rows].clone().requires_grad_(True) for t in (q, k, v))
    out = ctx.attention(ql, kl, vl)
    (out.float() * go[rows].float()).sum().backward()
    torch.cuda.synchronize()
    check_status(dev)
    for name, got, want in (("out", out, full[rows]), ("dq", ql.grad, qf.grad[rows]),
                            ("dk", kl.grad, kf.grad[rows]), ("dv", vl.grad, vf.grad[rows])):
        err = rel(got, want)
        assert err < 3e-2, f"ring attention {name} rel err {err}"

    # 2b. the same attention with the kernels reading peer tiles over NVLink
    from prism_cp_b200.parallel import layout as layout_mod
    layout_mod.CP_ATTENTION["impl"] = "peer"
    pctx = LocalLayout(Layout((Group(ranks, (0, 1)),), "zigzag"), alen, world, rank, dev, teams)
    qp, kp, vp = (t[rows].clone().requires_grad_(True) for t in (q, k, v))
    for _ in range(3):  # repeated calls cycle both heap halves and the done/ready protocol
        for t in (qp, kp, vp):
            t.grad = None
        outp = pctx.attention(qp, kp, vp)
        (outp.float() * go[rows].float()).sum().backward()
    torch.cuda.synchronize()
    check_status(dev)
    layout_mod.CP_ATTENTION["impl"] = "ring"
    assert type(pctx._cp_attn).__name__ == "PeerAttention"
    for name, got, want in (("out", outp, full[rows]), ("dq", qp.grad, qf.grad[rows]),
                            ("dk", kp.grad, kf.grad[rows]), ("dv", vp.grad, vf.grad[rows])):
        err = rel(got, want)
        assert err < 3e-2, f"peer attention {name} rel err {err}"

    # 3. chunkwise GDN CP on the GPU state kernels vs one GPU
    # sample 1 spans a rank boundary, so a rank holds a finished sample and a continuing one (the
    # identity pass then runs over the continuing first segment alone)
    glen = {0: 640 * world // 2, 1: 2560 * world // 2, 2: 640 * world // 2}
    gctx = LocalLayout(Layout((Group(ranks, (0, 1, 2)),), "contiguous"), glen, world, rank, dev, teams)
    Tg, H, dk, dv = sum(glen.values()), 4, 128, 256
    g2 = torch.Generator(device="cuda").manual_seed(5)
    qq = F.normalize(torch.randn(Tg, H, dk, device=dev, generator=g2), dim=-1)
    kk = F.normalize(torch.randn(Tg, H, dk, device=dev, generator=g2), dim=-1)
    vv = torch.randn(Tg, H, dv, device=dev, generator=g2)
    gg = -torch.rand(Tg, H, device=dev, generator=g2) * 0.2
    bb = torch.rand(Tg, H, device=dev, generator=g2)
    ins = [t.clone().requires_grad_(True) for t in (qq, kk, vv, gg, bb)]
    ref, _ = chunk_gated_delta_rule(*ins, ChunkLayout((glen[0], glen[1], glen[2]), dev))
    gout = torch.randn_like(ref)
    (ref * gout).sum().backward()
    rows = rows_of(gctx, {0: 0, 1: glen[0], 2: glen[0] + glen[1]})
    loc = [t[rows].clone().requires_grad_(True) for t in (qq, kk, vv, gg, bb)]
    o = gctx.delta_rule(*loc)
    (o * gout[rows]).sum().backward()
    torch.cuda.synchronize()
    # the CP path runs the bf16 fused kernels (dk 128, dv 256): the zero-start pass over every segment
    # and the identity pass over a continuing first segment; the oracle is fp32 on one GPU
    assert rel(o, ref[rows]) < 2e-2, f"GDN CP output {rel(o, ref[rows])}"
    for name, t, r in zip("qkvgb", loc, ins):
        assert rel(t.grad, r.grad[rows]) < 1e-1, f"GDN CP gradient d{name} {rel(t.grad, r.grad[rows])}"

    # 3b. the same with both passes on one prep (PRISM_GDN_SHARED_PREP)
    from prism_cp_b200.parallel import gdn_cp
    gdn_cp.SHARED_PREP = True
    try:
        sctx = LocalLayout(Layout((Group(ranks, (0, 1, 2)),), "contiguous"), glen, world, rank, dev, teams)
        loc2 = [t[rows].clone().requires_grad_(True) for t in (qq, kk, vv, gg, bb)]
        o2 = sctx.delta_rule(*loc2)
        (o2 * gout[rows]).sum().backward()
        torch.cuda.synchronize()
        check_status(dev)
    finally:
        gdn_cp.SHARED_PREP = False
    assert rel(o2, ref[rows]) < 2e-2, f"GDN CP (shared prep) output {rel(o2, ref[rows])}"
    for name, t, r in zip("qkvgb", loc2, ins):
        assert rel(t.grad, r.grad[rows]) < 1e-1, f"GDN CP (shared prep) gradient d{name} {rel(t.grad, r.grad[rows])}"

    # 4. tensor parallelism over all ranks (TP = world, CP = 1) on the sm_100a kernels vs one GPU
    from prism_cp_b200.models.config import HybridConfig
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.tensor import make_tp
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = HybridConfig(num_layers=4, hidden_size=512, ffn_hidden_size=1024, vocab_size=4096,
                       num_attention_heads=8, num_query_groups=4, kv_channels=128,
                       linear_num_key_heads=4, linear_key_head_dim=128, linear_value_head_dim=256, name="tp-check")
    batch = make_batch([1024, 512], cfg.vocab_size, seed=3)
    tpc = make_tp(world)
    tp_model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0, tp=tpc)
    tp_trainer = Trainer(tp_model, Teams(tp=tpc), dev, lr=1e-3)
    plan1 = uniform_plan(batch.lengths, 1, 1, 2048, cfg.pattern)
    tp_losses = [tp_trainer.train_step(batch, plan1).loss for _ in range(2)]
    ref_model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)

    class Solo:
        world, rank, initialized = 1, 0, False

        def team(self, ranks):
            return None

    ref_trainer = Trainer(ref_model, Solo(), dev, lr=1e-3)
    ref_losses = [ref_trainer.train_step(batch, plan1).loss for _ in range(2)]
    torch.cuda.synchronize()
    check_status(dev)
    for a_, b_ in zip(tp_losses, ref_losses):
        assert abs(a_ - b_) <= 2e-2 * abs(b_), f"TP loss {tp_losses} vs single GPU {ref_losses}"

    # 5. fused tensor-parallel GEMM + all-reduce over peer memory vs GEMM + NCCL all-reduce (fp32 oracle)
    from prism_cp_b200.parallel.tp_fused import FusedAllReduceGemm
    fused = FusedAllReduceGemm(dist.group.WORLD, dev)
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    for (M, N, K, b_mn) in [(1000, 2048, 512, False), (4096, 1024, 768, True), (384, 520, 64, False),
                            (8192, 2048, 1024, False), (1000, 2048, 512, False)]:
        a = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
        b = torch.randn(K, N, device=dev, generator=gen).to(torch.bfloat16) if b_mn else \
            torch.randn(N, K, device=dev, generator=gen).to(torch.bfloat16)
        got = fused(a, b, b_mn=b_mn)
        want = a.float() @ (b.float() if b_mn else b.float().t())
        dist.all_reduce(want)
        torch.cuda.synchronize()
        check_status(dev)
        assert rel(got, want) < 1e-2, f"fused GEMM+all-reduce {M}x{N}x{K} b_mn={b_mn}: {rel(got, want)}"
        same = got.clone()
        dist.broadcast(same, 0)
        assert torch.equal(same, got), f"fused GEMM+all-reduce results differ between ranks ({M}x{N}x{K})"
    fused.close()

    heap.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("MGPU_OK", flush=True)


if __name__ == "__main__":
    main()
