"""sm_100a kernels vs plain fp32 PyTorch references of the same ops."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _seed_and_status():
    torch.manual_seed(0)
    yield
    from prism_cp_b200.ops._lib import status
    torch.cuda.synchronize()
    assert int(status(torch.device(DEV, torch.cuda.current_device())).item()) == 0, "a device wait timed out"


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (304, 520, 200), (1024, 2048, 2048), (4096, 12320, 2048)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm(M, N, K, a_mn, b_mn):
    from prism_cp_b200.ops.gemm import matmul
    if (M, N, K) == (4096, 12320, 2048) and (a_mn or b_mn):
        pytest.skip("large case runs once")
    A = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    B = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    out = matmul(a, b, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2


def test_gemm_fp32_accumulate_and_rowscale():
    from prism_cp_b200.ops.gemm import matmul
    M, N, K = 384, 640, 256
    A = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    B = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    C = torch.randn(M, N, device=DEV, dtype=torch.float32)
    s = torch.rand(M, device=DEV, dtype=torch.float32)
    ref = C + (A.float() @ B.float().t()) * s[:, None]
    matmul(A, B, out=C, accumulate=True, row_scale=s)
    assert rel_err(C, ref) < 1e-3


# ------------------------------------------------------------------ norms
def test_rmsnorm_fwd_bwd():
    from prism_cp_b200.ops.norms import rms_norm
    x = torch.randn(1000, 2048, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(2048, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    y = rms_norm(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    yr.backward(g.float())
    assert rel_err(y, yr) < 1e-2
    assert rel_err(x.grad, xr.grad) < 2e-2
    assert rel_err(w.grad, wr.grad) < 2e-2


def test_gated_and_l2_norm():
    from prism_cp_b200.ops.norms import gated_rms_norm, l2_norm
    T, H, n = 333, 4, 256
    x = torch.randn(T, H * n, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    z = torch.randn(T, H * n, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(n, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    y = gated_rms_norm(x, z, w, H)
    g = torch.randn_like(y)
    y.backward(g)
    xr, zr, wr = (t.detach().float().requires_grad_(True) for t in (x, z, w))
    x3 = xr.view(T, H, n)
    yr = (x3 * torch.rsqrt(x3.pow(2).mean(-1, keepdim=True) + 1e-6) * wr * F.silu(zr.view(T, H, n))).view(T, -1)
    yr.backward(g.float())
    for a, b in ((y, yr), (x.grad, xr.grad), (z.grad, zr.grad), (w.grad, wr.grad)):
        assert rel_err(a, b) < 2e-2
    q = torch.randn(T, H * 128, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    yq = l2_norm(q, H)
    gq = torch.randn_like(yq)
    yq.backward(gq)
    qr = q.detach().float().requires_grad_(True)
    q3 = qr.view(T, H, 128)
    yqr = (q3 * torch.rsqrt(q3.pow(2).sum(-1, keepdim=True) + 1e-6)).view(T, -1)
    yqr.backward(gq.float())
    assert rel_err(yq, yqr) < 1e-2 and rel_err(q.grad, qr.grad) < 2e-2


# ------------------------------------------------------------------ elementwise
def test_rope_roundtrip_and_reference():
    from prism_cp_b200.ops.elementwise import _ref_rope, rope
    T, H, d = 500, 8, 128
    base = torch.randn(T, 3 * H * d, device=DEV, dtype=torch.bfloat16)
    x = base[:, H * d: 2 * H * d].detach().requires_grad_(True)
    pos = torch.randint(0, 40000, (T,), device=DEV, dtype=torch.int32)
    y = rope(x, pos, H, d)
    ref = _ref_rope(x.detach().float(), pos, H, d, 10000.0, False)
    assert rel_err(y, ref) < 1e-2
    g = torch.randn_like(y)
    y.backward(g)
    gref = _ref_rope(g.float(), pos, H, d, 10000.0, True)
    assert rel_err(x.grad, gref) < 1e-2


def test_conv1d_silu_fwd_bwd_with_halo():
    from prism_cp_b200.ops.elementwise import _ref_conv, causal_conv1d_silu
    T, C = 700, 384
    x = torch.randn(T, C, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (0.5 * torch.randn(C, 4, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    halo = torch.randn(3, C, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    cu = torch.tensor([0, 130, 131, 400, 700], device=DEV, dtype=torch.int32)
    y = causal_conv1d_silu(x, w, cu, halo)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr, hr = (t.detach().float().requires_grad_(True) for t in (x, w, halo))
    yr = _ref_conv(xr, wr, hr, cu.cpu())
    yr.backward(g.float())
    for a, b in ((y, yr), (x.grad, xr.grad), (w.grad, wr.grad), (halo.grad, hr.grad)):
        assert rel_err(a, b) < 2e-2


def test_swiglu():
    from prism_cp_b200.ops.elementwise import swiglu
    x = torch.randn(300, 2 * 3584, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    y = swiglu(x)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    a, b = xr.chunk(2, -1)
    yr = F.silu(a) * b
    yr.backward(g.float())
    assert rel_err(y, yr) < 1e-2 and rel_err(x.grad, xr.grad) < 2e-2


def test_head_cross_entropy():
    from prism_cp_b200.ops.cross_entropy import head_cross_entropy
    T, H, V = 3000, 512, 32000
    h = (0.5 * torch.randn(T, H, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    W = (0.05 * torch.randn(V, H, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    labels = torch.randint(0, V, (T,), device=DEV)
    wt = (torch.rand(T, device=DEV) > 0.3).float() / T
    loss, ce = head_cross_entropy(h, W, labels, wt, chunk=1024)
    loss.backward()
    hr, Wr = h.detach().float().requires_grad_(True), W.detach().float().requires_grad_(True)
    cer = F.cross_entropy(hr @ Wr.t(), labels, reduction="none")
    lr = (cer * wt).sum()
    lr.backward()
    assert abs(loss.item() - lr.item()) / abs(lr.item()) < 1e-2
    assert rel_err(ce, cer) < 1e-2
    assert rel_err(h.grad, hr.grad) < 3e-2
    assert rel_err(W.grad, Wr.grad) < 3e-2


def test_adamw_and_sumsq():
    from prism_cp_b200.ops._lib import lib
    n = 1_000_003
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m = torch.randn(n, device=DEV).abs() * 0.1
    v = torch.rand(n, device=DEV) * 0.1
    ss = torch.zeros(1, device=DEV)
    lib().sumsq_accumulate(g, ss)
    assert abs(ss.item() - g.pow(2).sum().item()) / g.pow(2).sum().item() < 1e-4
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    pb = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    lr, b1, b2, eps, wd, step, clip = 1e-3, 0.9, 0.95, 1e-8, 0.1, 3, 1.0
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    lib().adamw_step(p, g, m, v, pb, ss, clip, lr, b1, b2, eps, wd, bc1, bc2)
    coef = min(1.0, clip / (math.sqrt(ss.item()) + 1e-6))
    gg = g * coef
    mr = b1 * mr + (1 - b1) * gg
    vr = b2 * vr + (1 - b2) * gg * gg
    pr = pr - lr * ((mr / bc1) / ((vr / bc2).sqrt() + eps) + wd * pr)
    assert rel_err(p, pr) < 1e-5 and rel_err(m, mr) < 1e-5 and rel_err(v, vr) < 1e-5
    assert rel_err(pb, pr) < 1e-2


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("lens,causal", [((128,), True), ((1000, 37, 2100), True), ((256, 384), False)])
def test_attention_fwd_bwd(lens, causal):
    from prism_cp_b200.ops.attention import AttentionMeta, flash_attention, reference_attention
    Hq, Hkv, d = 8, 2, 128
    T = sum(lens)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * d, device=DEV, dtype=torch.bfloat16)
    q = qkv[:, :Hq * d].view(T, Hq, d).detach().requires_grad_(True)
    k = qkv[:, Hq * d:(Hq + Hkv) * d].view(T, Hkv, d).detach().requires_grad_(True)
    v = qkv[:, (Hq + Hkv) * d:].view(T, Hkv, d).detach().requires_grad_(True)
    meta = AttentionMeta(lens, lens, causal, torch.device(DEV))
    out, lse = flash_attention(q, k, v, meta)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref, lse_ref = reference_attention(qr, kr, vr, meta, d ** -0.5)
    assert rel_err(out, ref) < 2e-2
    assert (lse - lse_ref).abs().max().item() < 2e-2
    g = torch.randn_like(out)
    out.backward(g)
    ref.backward(g.float())
    assert rel_err(q.grad, qr.grad) < 3e-2
    assert rel_err(k.grad, kr.grad) < 3e-2
    assert rel_err(v.grad, vr.grad) < 3e-2


# ------------------------------------------------------------------ GDN
def test_gdn_chunk_matches_token_recurrence():
    from prism_cp_b200.ops.gdn import ChunkLayout, chunk_gated_delta_rule, naive_gated_delta_rule
    lens = (200, 64, 130)
    T, H, dk, dv = sum(lens), 2, 128, 256
    q = F.normalize(torch.randn(T, H, dk, device=DEV), dim=-1)
    k = F.normalize(torch.randn(T, H, dk, device=DEV), dim=-1)
    v = torch.randn(T, H, dv, device=DEV)
    g = -torch.rand(T, H, device=DEV) * 0.2
    beta = torch.rand(T, H, device=DEV)
    s0 = torch.randn(len(lens), H, dk, dv, device=DEV) * 0.1
    layout = ChunkLayout(lens, torch.device(DEV))
    o, fin = chunk_gated_delta_rule(q, k, v, g, beta, layout, initial_state=s0)
    ref, fin_ref = naive_gated_delta_rule(q.cpu(), k.cpu(), v.cpu(), g.cpu(), beta.cpu(), lens,
                                          initial_state=s0.cpu())
    assert rel_err(o.cpu(), ref) < 1e-4
    assert rel_err(fin.cpu(), fin_ref) < 1e-4


def test_gdn_chunk_gradients_vs_cpu():
    from prism_cp_b200.ops.gdn import ChunkLayout, chunk_gated_delta_rule
    lens = (150, 70)
    T, H, dk, dv = sum(lens), 2, 128, 64
    base = [F.normalize(torch.randn(T, H, dk), dim=-1), F.normalize(torch.randn(T, H, dk), dim=-1),
            torch.randn(T, H, dv), -torch.rand(T, H) * 0.2, torch.rand(T, H), torch.randn(2, H, dk, dv) * 0.1]
    grads = []
    for dev in ("cpu", DEV):
        ts = [b.detach().clone().to(dev).requires_grad_(True) for b in base]
        layout = ChunkLayout(lens, torch.device(dev))
        o, fin = chunk_gated_delta_rule(*ts[:5], layout, initial_state=ts[5])
        (o.pow(2).sum() + fin.sum()).backward()
        grads.append([t.grad.cpu() for t in ts])
    for a, b in zip(*grads):
        assert rel_err(b, a) < 1e-3


# ------------------------------------------------------------------ model
def test_model_step_gpu_matches_fp32_cpu_direction():
    from prism_cp_b200.models.config import HybridConfig
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.layout import LocalLayout, single_rank_layout
    cfg = HybridConfig(num_layers=4, hidden_size=256, ffn_hidden_size=512, vocab_size=4096,
                       num_attention_heads=4, num_query_groups=2, kv_channels=128,
                       linear_num_key_heads=2, linear_key_head_dim=128, linear_value_head_dim=128)
    lengths = {0: 300, 1: 212}
    T = sum(lengths.values())
    tokens = torch.randint(0, cfg.vocab_size, (T,))
    labels = torch.randint(0, cfg.vocab_size, (T,))
    wt = torch.full((T,), 1.0 / T)
    losses = []
    for dev, dtype in (("cpu", torch.float32), (DEV, torch.bfloat16)):
        model = HybridModel(cfg, dtype=dtype, device=dev, seed=0)
        lay = LocalLayout(single_rank_layout(lengths), lengths, 1, 0, torch.device(dev))
        ctxs = [lay if s == "*" else LocalLayout(single_rank_layout(lengths, "contiguous"), lengths, 1, 0,
                                                  torch.device(dev)) for s in cfg.pattern]
        loss, _ = model(tokens.to(dev), labels.to(dev), wt.to(dev), ctxs)
        loss.backward()
        losses.append(loss.item())
        assert all(p.grad is None or torch.isfinite(p.grad).all() for p in model.parameters())
    assert abs(losses[0] - losses[1]) / abs(losses[0]) < 2e-2


def test_recomputed_layers_on_cuda_match_stored_activations():
    """Per-layer recompute on the CUDA kernels (GDN fused rule, attention, GEMMs): the loss and
    every gradient equal the run that keeps its activations."""
    from prism_cp_b200.models.config import HybridConfig
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = HybridConfig(num_layers=4, hidden_size=256, ffn_hidden_size=512, vocab_size=4096,
                       num_attention_heads=4, num_query_groups=2, kv_channels=128,
                       linear_num_key_heads=2, linear_key_head_dim=128, linear_value_head_dim=256)
    dev = torch.device(DEV, torch.cuda.current_device())
    out = {}
    for limit in (None, 256):
        model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)
        batch = make_batch([640, 384], cfg.vocab_size, seed=2)
        plan = uniform_plan(batch.lengths, 1, 1, 1024, cfg.pattern)
        tr = Trainer(model, Teams(1), dev, recompute_tokens=limit)
        tr.flat.zero_grad()
        loss = tr.forward_backward(batch.lengths, plan, [h.to(dev) for h in tr.prepare(batch, plan)])
        tr.flat.fold_param_grads()
        torch.cuda.synchronize()
        out[limit] = (float(loss), tr.flat.grad.clone())
    assert abs(out[None][0] - out[256][0]) <= 1e-3 * abs(out[None][0])
    g0, g1 = out[None][1], out[256][1]
    assert torch.isfinite(g1).all()
    assert ((g0 - g1).norm() / g0.norm()).item() < 1e-2


def test_overlapped_gradient_and_parameter_sync_on_cuda_match_serial():
    """Bucketed reduce-scatter during the backward and parameter all-gather on a side stream during
    the next forward (forward pre-hooks wait per bucket) give the same three steps as the serial
    single-bucket sync."""
    from prism_cp_b200.models.config import HybridConfig
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = HybridConfig(num_layers=4, hidden_size=256, ffn_hidden_size=512, vocab_size=4096,
                       num_attention_heads=4, num_query_groups=2, kv_channels=128,
                       linear_num_key_heads=2, linear_key_head_dim=128, linear_value_head_dim=256)
    dev = torch.device(DEV, torch.cuda.current_device())
    out = []
    for overlap in (False, True):
        model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)
        batch = make_batch([640, 384], cfg.vocab_size, seed=2)
        plan = uniform_plan(batch.lengths, 1, 1, 1024, cfg.pattern)
        tr = Trainer(model, Teams(1), dev, overlap_grad_reduce=overlap, overlap_param_gather=overlap,
                     bucket_bytes=1 << 20)
        if overlap:
            assert len(tr.flat.buckets) > 2
        losses = [tr.train_step(batch, plan).loss for _ in range(3)]
        tr.optimizer.wait_parameters()
        torch.cuda.synchronize()
        out.append((losses, torch.cat([p.detach().float().reshape(-1) for p in model.parameters()])))
    (l0, p0), (l1, p1) = out
    assert l0 == pytest.approx(l1, rel=2e-3)
    assert ((p0 - p1).norm() / p0.norm()).item() < 1e-3


@pytest.mark.parametrize("j", [5, 200, 511])
def test_cuda_model_is_causal(j):
    """Changing token j changes no hidden state before position j on the CUDA kernels (GEMMs,
    conv, fused GDN chunks, flash attention); states from j on do change."""
    from prism_cp_b200.models.config import HybridConfig
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.layout import LocalLayout, single_rank_layout
    cfg = HybridConfig(num_layers=4, hidden_size=256, ffn_hidden_size=512, vocab_size=4096,
                       num_attention_heads=4, num_query_groups=2, kv_channels=128,
                       linear_num_key_heads=2, linear_key_head_dim=128, linear_value_head_dim=256)
    lengths = {0: 640}
    dev = torch.device(DEV, torch.cuda.current_device())
    model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)
    lay = LocalLayout(single_rank_layout(lengths), lengths, 1, 0, dev)
    flat = LocalLayout(single_rank_layout(lengths, "contiguous"), lengths, 1, 0, dev)
    ctxs = [lay if s == "*" else flat for s in cfg.pattern]
    tokens = torch.randint(0, cfg.vocab_size, (640,), generator=torch.Generator().manual_seed(4)).to(dev)
    other = tokens.clone()
    other[j] = (other[j] + 1) % cfg.vocab_size
    with torch.no_grad():
        a = model.run_layers(model.embed(tokens), ctxs)
        b = model.run_layers(model.embed(other), ctxs)
    torch.cuda.synchronize()
    assert torch.equal(a[:j], b[:j]), "a hidden state before the changed token moved"
    assert not torch.equal(a[j:], b[j:])


def test_repeated_random_batch_is_memorised_not_leaked():
    """The benchmark trains on one synthetic batch of uniform random tokens every step, and its loss
    falls far below ln(vocab). That is memorisation of the repeated batch, not a view of the future:
    the same trained model scores an unseen random batch at about ln(vocab)."""
    import math
    from prism_cp_b200.models.config import HybridConfig
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = HybridConfig(num_layers=4, hidden_size=256, ffn_hidden_size=512, vocab_size=4096,
                       num_attention_heads=4, num_query_groups=2, kv_channels=128,
                       linear_num_key_heads=2, linear_key_head_dim=128, linear_value_head_dim=256)
    dev = torch.device(DEV, torch.cuda.current_device())
    model = HybridModel(cfg, dtype=torch.bfloat16, device=dev, seed=0)
    tr = Trainer(model, Teams(1), dev, lr=3e-3, warmup_steps=0)
    seen = make_batch([512, 512], cfg.vocab_size, seed=11)
    unseen = make_batch([512, 512], cfg.vocab_size, seed=12)
    plan = uniform_plan(seen.lengths, 1, 1, 1024, cfg.pattern)
    first = tr.train_step(seen, plan).loss
    for _ in range(40):
        last = tr.train_step(seen, plan).loss
    with torch.no_grad():
        from prism_cp_b200.runtime.executor import MicrobatchRun
        inputs = tr.prepare(unseen, plan)[0].to(dev)
        run = MicrobatchRun(plan.microbatches[0], unseen.lengths, tr.cache)
        held_out, _ = run.forward(model, inputs.tokens, inputs.labels, inputs.weights)
    ln_v = math.log(cfg.vocab_size)
    assert abs(first - ln_v) < 1.0
    assert last < 0.5 * ln_v, (first, last)
    assert float(held_out) > 0.9 * ln_v, float(held_out)


# ------------------------------------------------------------------ bounded device waits
def test_a_device_wait_that_runs_out_reports_an_error_and_the_context_survives():
    """A flag nothing sets: the bounded wait gives up after its limit, records an error status the
    host reads, and the CUDA context keeps working (no trap, no hang)."""
    import time
    from prism_cp_b200.ops._lib import check_status, lib, status
    dev = torch.device(DEV, torch.cuda.current_device())
    flags = torch.zeros(8, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    lib().symm_wait(flags.data_ptr(), 0, 1, 1, status(dev), 1_000_000_000)  # a flag nothing sets: 1 s limit
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 0.8 < waited < 60, waited
    # a gather queued behind the failed wait copies nothing (no stale rows reach the output)
    src = torch.arange(64 * 8, dtype=torch.float32, device=dev).view(64, 8)
    dst = torch.full((64, 8), -1.0, device=dev)
    bases = torch.tensor([src.data_ptr()], dtype=torch.int64, device=dev)
    routes = torch.tensor([[0, 0, 0, 64]], dtype=torch.int64, device=dev)
    block_route = torch.zeros(2, dtype=torch.int64, device=dev)
    block_row0 = torch.tensor([0, 32], dtype=torch.int64, device=dev)
    lib().symm_gather_rows(bases, routes, block_route, block_row0, 32, 32, dst, status(dev))
    torch.cuda.synchronize()
    assert bool((dst == -1.0).all())
    with pytest.raises(RuntimeError, match="timed out"):
        check_status(dev)
    # with the status cleared the same gather copies every row
    lib().symm_gather_rows(bases, routes, block_route, block_row0, 32, 32, dst, status(dev))
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
    a = torch.randn(256, 256, device=dev)
    assert torch.allclose(a @ torch.eye(256, device=dev), a)
