"""Context-parallel plumbing on CPU ranks (gloo): every distributed path vs a one-process oracle."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, queue, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.manual_seed(0)
        fn(rank, world, *args)
        dist.barrier()
        queue.put((rank, None))
    except Exception:  # pragma: no cover - reported to the parent
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world, *args, timeout=240):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, queue, args)) for r in range(world)]
    for p in procs:
        p.start()
    errors = []
    for _ in procs:
        rank, err = queue.get(timeout=timeout)
        if err:
            errors.append(f"rank {rank}:\n{err}")
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert not errors, "\n".join(errors)


def _close(a, b, tol=1e-4):
    err = ((a.double() - b.double()).norm() / (b.double().norm() + 1e-12)).item()
    assert err < tol, f"relative error {err}"


# ------------------------------------------------------------------ ring attention
def _ring_case(rank, world):
    from prism_cp_b200.ops.attention import AttentionMeta, reference_attention
    from prism_cp_b200.parallel.layout import LocalLayout
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.joint.ir import Group, Layout
    lengths = {0: 64, 1: 32 * world // 2 * 2}
    lay = Layout((Group(tuple(range(world)), (0, 1)),), "zigzag")
    ctx = LocalLayout(lay, lengths, world, rank, torch.device("cpu"), Teams(world))
    g = torch.Generator().manual_seed(3)
    T = sum(lengths.values())
    Hq, Hkv, d = 4, 2, 16
    q = torch.randn(T, Hq, d, generator=g, dtype=torch.float64)
    k = torch.randn(T, Hkv, d, generator=g, dtype=torch.float64)
    v = torch.randn(T, Hkv, d, generator=g, dtype=torch.float64)
    go = torch.randn(T, Hq, d, generator=g, dtype=torch.float64)
    # global oracle
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    meta = AttentionMeta((lengths[0], lengths[1]), (lengths[0], lengths[1]), True, torch.device("cpu"))
    ref, _ = reference_attention(qr, kr, vr, meta, d ** -0.5)
    (ref * go).sum().backward()
    # local rows of this rank in zigzag order
    offs = {0: 0, 1: lengths[0]}
    rows = torch.tensor([offs[s] + b + j for s, b, _, c in ctx.spans for j in range(c)])
    ql, kl, vl = (t[rows].clone().requires_grad_(True) for t in (q, k, v))
    out = ctx.attention(ql, kl, vl)
    _close(out, ref[rows].detach(), 1e-5)
    (out * go[rows]).sum().backward()
    _close(ql.grad, qr.grad[rows], 1e-5)
    _close(kl.grad, kr.grad[rows], 1e-5)
    _close(vl.grad, vr.grad[rows], 1e-5)


@pytest.mark.parametrize("world", [2, 4])
def test_zigzag_ring_attention_matches_full_attention(world):
    run_ranks(_ring_case, world)


# ------------------------------------------------------------------ GDN CP
def _gdn_case(rank, world, lengths):
    import torch.nn.functional as F
    from prism_cp_b200.ops.gdn import ChunkLayout, chunk_gated_delta_rule
    from prism_cp_b200.parallel.layout import LocalLayout
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.joint.ir import Group, Layout
    lengths = dict(lengths)
    lay = Layout((Group(tuple(range(world)), tuple(sorted(lengths))),), "contiguous")
    ctx = LocalLayout(lay, lengths, world, rank, torch.device("cpu"), Teams(world))
    g = torch.Generator().manual_seed(5)
    T = sum(lengths.values())
    H, dk, dv = 2, 16, 8
    q = F.normalize(torch.randn(T, H, dk, generator=g, dtype=torch.float64), dim=-1)
    k = F.normalize(torch.randn(T, H, dk, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(T, H, dv, generator=g, dtype=torch.float64)
    gl = -torch.rand(T, H, generator=g, dtype=torch.float64) * 0.3
    beta = torch.rand(T, H, generator=g, dtype=torch.float64)
    go = torch.randn(T, H, dv, generator=g, dtype=torch.float64)
    ins = [t.clone().requires_grad_(True) for t in (q, k, v, gl, beta)]
    full = ChunkLayout(tuple(lengths[s] for s in sorted(lengths)), torch.device("cpu"))
    ref, _ = chunk_gated_delta_rule(*ins, full)
    (ref * go).sum().backward()
    offs, acc = {}, 0
    for s in sorted(lengths):
        offs[s] = acc
        acc += lengths[s]
    rows = torch.tensor([offs[s] + b + j for s, b, _, c in ctx.spans for j in range(c)])
    loc = [t[rows].clone().requires_grad_(True) for t in (q, k, v, gl, beta)]
    out = ctx.delta_rule(*loc)
    _close(out, ref[rows].detach(), 1e-5)
    (out * go[rows]).sum().backward()
    for a, b in zip(loc, ins):
        _close(a.grad, b.grad[rows], 1e-5)


@pytest.mark.parametrize("world,lengths", [
    (2, ((0, 200), (1, 120))),            # sample 0 continues from rank 0 to rank 1
    (4, ((0, 448), (1, 64))),             # sample 0 spans ranks 0-3: ranks 1 and 2 pass the state through
    (2, ((0, 200), (1, 120), (2, 90))),   # rank 1: a continuing first segment followed by a whole sample
    (4, ((0, 96), (1, 380), (2, 36))),    # sample 1 from rank 0 through rank 3, starting mid-rank
])
def test_gdn_chunkwise_cp_matches_single_rank(world, lengths):
    run_ranks(_gdn_case, world, lengths)


def _conv_case(rank, world):
    from prism_cp_b200.ops.elementwise import causal_conv1d_silu
    from prism_cp_b200.parallel.layout import LocalLayout
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.joint.ir import Group, Layout
    lengths = {0: 70, 1: 2, 2: 8}  # the 2-token sample starts just before a rank boundary
    lay = Layout((Group(tuple(range(world)), (0, 1, 2)),), "contiguous")
    ctx = LocalLayout(lay, lengths, world, rank, torch.device("cpu"), Teams(world))
    g = torch.Generator().manual_seed(9)
    T, C = 80, 6
    x = torch.randn(T, C, generator=g, dtype=torch.float64)
    w = torch.randn(C, 4, generator=g, dtype=torch.float64)
    go = torch.randn(T, C, generator=g, dtype=torch.float64)
    xr = x.clone().requires_grad_(True)
    ref = causal_conv1d_silu(xr, w, torch.tensor([0, 70, 72, 80]))
    (ref * go).sum().backward()
    offs = {0: 0, 1: 70, 2: 72}
    rows = torch.tensor([offs[s] + b + j for s, b, _, c in ctx.spans for j in range(c)])
    xl = x[rows].clone().requires_grad_(True)
    out = ctx.conv(xl, w)
    _close(out, ref[rows].detach(), 1e-6)
    (out * go[rows]).sum().backward()
    _close(xl.grad, xr.grad[rows], 1e-6)


def test_conv_halo_across_ranks():
    run_ranks(_conv_case, 4)


# ------------------------------------------------------------------ transport
def _transport_case(rank, world):
    from prism_cp_b200.parallel.layout import LocalLayout
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.parallel.transport import move
    from prism_cp_b200.planner.joint.ir import Group, Layout
    lengths = {0: 32, 1: 16, 2: 16}
    teams = Teams(world)
    a = LocalLayout(Layout((Group((0, 1), (0, 1, 2)),), "zigzag"), lengths, world, rank, "cpu", teams)
    b = LocalLayout(Layout((Group((0,), (0,)), Group((1,), (1, 2))), "contiguous"), lengths, world, rank, "cpu",
                    teams)
    code = {0: 0, 1: 1000, 2: 2000}
    src = torch.tensor([[code[s] + b0 + j] for s, b0, _, c in a.spans for j in range(c)], dtype=torch.float64)
    src.requires_grad_(True)
    got = move(src, a, b)
    want = torch.tensor([[code[s] + b0 + j] for s, b0, _, c in b.spans for j in range(c)], dtype=torch.float64)
    assert torch.equal(got.detach(), want)
    (got * got).sum().backward()  # inverse route brings every gradient home
    assert torch.equal(src.grad, 2 * src.detach())


def test_transport_is_an_exact_permutation_with_inverse_backward():
    run_ranks(_transport_case, 2)


# ------------------------------------------------------------------ end-to-end tiny model
def _tiny_model_case(rank, world, steps):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.joint.ir import Group, Layout, Microbatch, Plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    gen = torch.Generator().manual_seed(0)
    cut = 4 * int(torch.randint(64, 448, (1,), generator=gen))      # uniform-random document boundary
    lengths = [cut, 2048 - cut]
    batch = make_batch(lengths, cfg.vocab_size, seed=0)
    gdn = Layout((Group((0, 1), (0, 1)),), "contiguous")
    gqa = Layout((Group((0,), (0,)), Group((1,), (1,))), "zigzag")
    layers = tuple((gdn, gdn) if c == "G" else (gqa, gqa) for c in cfg.pattern)
    plan = Plan(2, cfg.pattern, (Microbatch(gqa, layers),))
    model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
    trainer = Trainer(model, Teams(world), torch.device("cpu"), lr=1e-3, weight_decay=0.1)
    # gradients of the first microbatch, summed over the team
    trainer.flat.zero_grad()
    trainer.forward_backward(batch.lengths, plan, trainer.prepare(batch, plan))
    trainer.flat.fold_param_grads()
    grads = trainer.flat.grad.clone()
    dist.all_reduce(grads)
    losses, norms = [], []
    for _ in range(steps):
        res = trainer.train_step(batch, plan)
        losses.append(res.loss)
        norms.append(float(trainer.optimizer.sumsq.sqrt()))
    if rank == 0:
        # single-process oracle: the same model, data and optimizer at CP = 1
        ref_model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
        one = Layout((Group((0,), (0, 1)),), "zigzag")
        ref_plan = Plan(1, cfg.pattern, (Microbatch(one, tuple((one.with_mode("contiguous"),) * 2 if c == "G"
                                                                  else (one, one) for c in cfg.pattern)),))

        class Solo:
            world, rank, initialized = 1, 0, False

            def team(self, ranks):
                return None

        ref_tr = Trainer(ref_model, Solo(), torch.device("cpu"), lr=1e-3, weight_decay=0.1)
        ref_tr.flat.zero_grad()
        ref_tr.forward_backward(batch.lengths, ref_plan, ref_tr.prepare(batch, ref_plan))
        ref_tr.flat.fold_param_grads()
        n = min(grads.numel(), ref_tr.flat.grad.numel())  # tail padding depends on the world size
        _close(grads[:n], ref_tr.flat.grad[:n], 1e-4)
        for i in range(steps):
            r = ref_tr.train_step(batch, ref_plan)
            # fp32: the CP run re-chunks the GDN recurrence at rank boundaries
            assert abs(r.loss - losses[i]) / abs(r.loss) < 1e-4, (r.loss, losses[i])
            assert abs(float(ref_tr.optimizer.sumsq.sqrt()) - norms[i]) / norms[i] < 1e-3


def test_tiny_hybrid_cp2_matches_cp1_over_two_steps():
    run_ranks(_tiny_model_case, 2, 2, timeout=600)


# ------------------------------------------------------------------ tensor parallel
def _tp_case(rank, world, tp, steps):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.parallel.tensor import make_tp
    from prism_cp_b200.planner.joint.ir import Group, Layout, Microbatch, Plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    lengths = [1280, 768]
    batch = make_batch(lengths, cfg.vocab_size, seed=1)
    tpc = make_tp(tp)
    L = world // tp
    if L == 2:
        gdn = Layout((Group((0, 1), (0, 1)),), "contiguous")
        gqa = Layout((Group((0,), (0,)), Group((1,), (1,))), "zigzag")
    else:
        gdn = Layout((Group((0,), (0, 1)),), "contiguous")
        gqa = Layout((Group((0,), (0, 1)),), "zigzag")
    layers = tuple((gdn, gdn) if c == "G" else (gqa, gqa) for c in cfg.pattern)
    plan = Plan(L, cfg.pattern, (Microbatch(gqa, layers),))
    model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0, tp=tpc)
    trainer = Trainer(model, Teams(tp=tpc), torch.device("cpu"), lr=1e-3, weight_decay=0.1)
    losses, norms = [], []
    for _ in range(steps):
        res = trainer.train_step(batch, plan)
        losses.append(res.loss)
        norms.append(float(trainer.optimizer.sumsq.sqrt()))
    if rank == 0:
        ref_model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
        one = Layout((Group((0,), (0, 1)),), "zigzag")
        ref_plan = Plan(1, cfg.pattern, (Microbatch(one, tuple((one.with_mode("contiguous"),) * 2 if c == "G"
                                                                  else (one, one) for c in cfg.pattern)),))

        class Solo:
            world, rank, initialized = 1, 0, False

            def team(self, ranks):
                return None

        ref_tr = Trainer(ref_model, Solo(), torch.device("cpu"), lr=1e-3, weight_decay=0.1)
        ref_losses, ref_norms = [], []
        for _ in range(steps):
            r = ref_tr.train_step(batch, ref_plan)
            ref_losses.append(r.loss)
            ref_norms.append(float(ref_tr.optimizer.sumsq.sqrt()))
        for a, b in zip(losses, ref_losses):
            assert abs(a - b) <= 1e-4 * abs(b), (losses, ref_losses)
        for a, b in zip(norms, ref_norms):
            assert abs(a - b) <= 1e-4 * abs(b), (norms, ref_norms)


def test_tensor_parallel_tp2_matches_single_process():
    run_ranks(_tp_case, 2, 2, 2, timeout=600)


def test_tensor_parallel_tp2_cp2_matches_single_process():
    run_ranks(_tp_case, 4, 2, 2, timeout=900)


# ------------------------------------------------------------------ pipeline parallel (1F1B)
def _pp_case(rank, world, pp, steps):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.pipeline import PipelineTrainer, make_stage
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    ws = world // pp
    batch = make_batch([1024, 512, 512, 256, 256], cfg.vocab_size, seed=2)
    plan = uniform_plan(batch.lengths, ws, ws, 1024 // ws, cfg.pattern)
    assert len(plan.microbatches) >= 2
    info = make_stage(pp, cfg.num_layers)
    model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0,
                        layers=range(info.first_layer, info.first_layer + info.num_layers),
                        pre_process=info.stage == 0, post_process=info.stage == pp - 1)
    trainer = PipelineTrainer(model, info, torch.device("cpu"), lr=1e-3, weight_decay=0.1)
    losses, norms = [], []
    for _ in range(steps):
        res = trainer.train_step(batch, plan)
        losses.append(res.loss)
        norms.append(float(trainer.optimizer.sumsq.sqrt()))
        assert 0.0 <= res.extra["bubble_fraction"] <= 1.0
    if rank == 0:
        ref_model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
        ref_plan = uniform_plan(batch.lengths, 1, 1, 1024, cfg.pattern)

        class Solo:
            world, rank, initialized = 1, 0, False

            def team(self, ranks):
                return None

        ref_tr = Trainer(ref_model, Solo(), torch.device("cpu"), lr=1e-3, weight_decay=0.1)
        ref_losses, ref_norms = [], []
        for _ in range(steps):
            r = ref_tr.train_step(batch, ref_plan)
            ref_losses.append(r.loss)
            ref_norms.append(float(ref_tr.optimizer.sumsq.sqrt()))
        for a, b in zip(losses, ref_losses):
            assert abs(a - b) <= 1e-4 * abs(b), (losses, ref_losses)
        for a, b in zip(norms, ref_norms):
            assert abs(a - b) <= 1e-4 * abs(b), (norms, ref_norms)


def test_pipeline_1f1b_pp2_matches_single_process():
    run_ranks(_pp_case, 2, 2, 2, timeout=600)


def test_pipeline_1f1b_pp2_cp2_matches_single_process():
    run_ranks(_pp_case, 4, 2, 2, timeout=900)


# ------------------------------------------------------------------ logical numerics gate
def _logical_case(rank, world, ref_dir):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.joint.ir import Group, Layout, Microbatch, Plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.numerics import LogicalNumerics
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    batch = make_batch([1152, 896], cfg.vocab_size, seed=4)
    if rank == 0:
        # reference: one process, CP = 1, writes every logical sample
        one = Layout((Group((0,), (0, 1)),), "zigzag")
        ref_plan = Plan(1, cfg.pattern, (Microbatch(one, tuple((one.with_mode("contiguous"),) * 2 if c == "G"
                                                                  else (one, one) for c in cfg.pattern)),))

        class Solo:
            world, rank, initialized = 1, 0, False

            def team(self, ranks):
                return None

        gate = LogicalNumerics(ref_dir, mode="write", steps=1, distributed=False)
        ref = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Solo(), torch.device("cpu"),
                      logical=gate)
        ref.train_step(batch, ref_plan)
    dist.barrier()
    # GDN layers at CP = 2 (contiguous), GQA at CP = 2 (zigzag): rows move between layouts
    gdn = Layout((Group((0, 1), (0, 1)),), "contiguous")
    gqa = Layout((Group((0, 1), (0, 1)),), "zigzag")
    plan = Plan(2, cfg.pattern, (Microbatch(gqa, tuple((gdn, gdn) if c == "G" else (gqa, gqa)
                                                       for c in cfg.pattern)),))
    gate = LogicalNumerics(ref_dir, mode="read", steps=1, rank=rank)
    tr = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Teams(world), torch.device("cpu"),
                 logical=gate)
    tr.train_step(batch, plan)
    assert not gate.failures


def test_logical_gate_cp2_matches_cp1_reference(tmp_path):
    run_ranks(_logical_case, 2, str(tmp_path))


# ------------------------------------------------------------------ the benchmark's layout at 4 and 8 ranks
def _wide_cp_case(rank, world):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    lengths = [256 * world * 2, 256 * world]      # every sequence splits into whole zigzag chunks
    batch = make_batch(lengths, cfg.vocab_size, seed=6)
    plan = uniform_plan(batch.lengths, world, world, 256 * 3, cfg.pattern)   # CP = world, as bench.py
    tr = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Teams(world), torch.device("cpu"),
                 lr=1e-3)
    losses = [tr.train_step(batch, plan).loss for _ in range(2)]
    if rank == 0:
        ref_plan = uniform_plan(batch.lengths, 1, 1, sum(lengths), cfg.pattern)

        class Solo:
            world, rank, initialized = 1, 0, False

            def team(self, ranks):
                return None

        ref = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Solo(), torch.device("cpu"),
                      lr=1e-3)
        ref_losses = [ref.train_step(batch, ref_plan).loss for _ in range(2)]
        for a, b in zip(losses, ref_losses):
            assert abs(a - b) <= 1e-4 * abs(b), (losses, ref_losses)


@pytest.mark.parametrize("world", [4, 8])
def test_bench_layout_cp_world_matches_cp1(world):
    run_ranks(_wide_cp_case, world, timeout=600)


# ------------------------------------------------------------------ heterogeneous CP inside one microbatch
def _mixed_case(rank, world):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.joint.ir import Group, Layout, Microbatch, Plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    batch = make_batch([1024, 384, 256], cfg.vocab_size, seed=8)
    # attention: sample 0 at CP = 2 (zigzag) beside samples 1 and 2 at CP = 1, all in one microbatch;
    # GDN: all three samples at CP = 4 (contiguous); every GDN <-> GQA boundary reshards
    gqa = Layout((Group((0, 1), (0,)), Group((2,), (1,)), Group((3,), (2,))), "zigzag")
    gdn = Layout((Group((0, 1, 2, 3), (0, 1, 2)),), "contiguous")
    plan = Plan(4, cfg.pattern, (Microbatch(gqa, tuple((gdn, gdn) if c == "G" else (gqa, gqa)
                                                       for c in cfg.pattern)),))
    tr = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Teams(world), torch.device("cpu"),
                 lr=1e-3, audit=True)
    losses = [tr.train_step(batch, plan).loss for _ in range(2)]
    # tokenwise operators ran once per microbatch over all segments (CP2 + CP1 + CP1 attention teams)
    assert tr.fusion.calls and all(v == 1 for v in tr.fusion.calls.values()), tr.fusion.calls
    assert tr.last_packet["forwards"] == tr.last_packet["backwards"] == 1
    if rank == 0:
        one = Layout((Group((0,), (0, 1, 2)),), "zigzag")
        ref_plan = Plan(1, cfg.pattern, (Microbatch(one, tuple((one.with_mode("contiguous"),) * 2 if c == "G"
                                                                  else (one, one) for c in cfg.pattern)),))

        class Solo:
            world, rank, initialized = 1, 0, False

            def team(self, ranks):
                return None

        ref = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Solo(), torch.device("cpu"),
                      lr=1e-3)
        ref_losses = [ref.train_step(batch, ref_plan).loss for _ in range(2)]
        for a, b in zip(losses, ref_losses):
            assert abs(a - b) <= 1e-4 * abs(b), (losses, ref_losses)


def test_heterogeneous_cp_in_one_microbatch_matches_cp1():
    run_ranks(_mixed_case, 4, timeout=600)


# ------------------------------------------------------------------ pipeline checkpoint / resume
def _pp_resume_case(rank, world, ck):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime import checkpoint
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.pipeline import PipelineTrainer, make_stage
    cfg = hybrid_tiny()
    pp = world
    batch = make_batch([512, 256, 256], cfg.vocab_size, seed=3)
    plan = uniform_plan(batch.lengths, 1, 1, 512, cfg.pattern)
    info = make_stage(pp, cfg.num_layers)

    def fresh():
        model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0,
                            layers=range(info.first_layer, info.first_layer + info.num_layers),
                            pre_process=info.stage == 0, post_process=info.stage == pp - 1)
        return PipelineTrainer(model, info, torch.device("cpu"), lr=1e-3)

    straight = fresh()
    want = [straight.train_step(batch, plan).loss for _ in range(3)]
    first = fresh()
    for _ in range(2):
        first.train_step(batch, plan)
    checkpoint.save(first, ck, plan_cursor=2)
    dist.barrier()
    resumed = fresh()
    cursor = checkpoint.load(resumed, checkpoint.latest(ck))
    assert cursor == 2 and resumed.optimizer.step_count == 2
    got = resumed.train_step(batch, plan).loss
    assert abs(got - want[2]) <= 1e-5 * abs(want[2]), (got, want)


def test_pipeline_checkpoint_resume_matches_uninterrupted_run(tmp_path):
    run_ranks(_pp_resume_case, 2, str(tmp_path / "ck"))


def _tp_resume_case(rank, world, ck):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.parallel.tensor import make_tp
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime import checkpoint
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    batch = make_batch([512, 256, 256], cfg.vocab_size, seed=3)
    plan = uniform_plan(batch.lengths, 1, 1, 1024, cfg.pattern)
    tpc = make_tp(world)

    def fresh():
        return Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0, tp=tpc), Teams(tp=tpc),
                       torch.device("cpu"), lr=1e-3)

    straight = fresh()
    want = [straight.train_step(batch, plan).loss for _ in range(3)]
    first = fresh()
    for _ in range(2):
        first.train_step(batch, plan)
    checkpoint.save(first, ck, plan_cursor=2)
    dist.barrier()
    resumed = fresh()
    assert checkpoint.load(resumed, checkpoint.latest(ck)) == 2
    got = resumed.train_step(batch, plan).loss
    assert abs(got - want[2]) <= 1e-5 * abs(want[2]), (got, want)


def test_tensor_parallel_checkpoint_resume_matches_uninterrupted_run(tmp_path):
    run_ranks(_tp_resume_case, 2, str(tmp_path / "ck"))


def _pp_records_case(rank, world, out):
    import json
    from pathlib import Path
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime import records
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.pipeline import PipelineTrainer, make_stage
    cfg = hybrid_tiny()
    batch = make_batch([512, 256, 256], cfg.vocab_size, seed=3)
    plan = uniform_plan(batch.lengths, 1, 1, 512, cfg.pattern)
    info = make_stage(world, cfg.num_layers)
    model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0,
                        layers=range(info.first_layer, info.first_layer + info.num_layers),
                        pre_process=info.stage == 0, post_process=info.stage == world - 1)
    tr = PipelineTrainer(model, info, torch.device("cpu"), lr=1e-3, records=out)
    for _ in range(3):
        tr.train_step(batch, plan)
    dist.barrier()
    if rank == 0:
        rows = [json.loads(x) for x in (Path(out) / "steps_rank1.jsonl").read_text().splitlines()]
        assert [r["step"] for r in rows] == [1, 2, 3] and rows[0]["pipeline"]["stage"] == 1
        manifest = {"input_tokens": batch.total_tokens, "loss_tokens": batch.loss_tokens}
        summary = records.summarize_records(out, manifest, 3, [2, 3], len(plan.microbatches), world=world)
        assert summary["status"] == "complete", summary


def test_pipeline_step_records_summarize_as_complete(tmp_path):
    run_ranks(_pp_records_case, 2, str(tmp_path / "rec"))
