"""Fused sm_100a chunked gated delta rule (csrc/gdn_chunk.cu) against fp32/fp64 PyTorch oracles."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _inputs(lens, H, dv, seed, with_state):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = F.normalize(torch.randn(T, H, 128, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(T, H, 128, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(T, H, dv, generator=g).to(torch.bfloat16)
    gl = -torch.rand(T, H, generator=g) * 0.3
    beta = torch.rand(T, H, generator=g)
    s0 = torch.randn(len(lens), H, 128, dv, generator=g) * 0.1 if with_state else None
    return q, k, v, gl, beta, s0


@pytest.mark.parametrize("lens,dv,with_state", [((150, 70, 300), 128, False), ((256, 64, 200), 256, True),
                                                ((1000,), 256, False)])
def test_fused_forward_matches_token_recurrence(lens, dv, with_state):
    from prism_cp_b200.ops._lib import check_status
    from prism_cp_b200.ops.gdn import ChunkLayout, fused_gated_delta_rule, naive_gated_delta_rule
    q, k, v, gl, beta, s0 = _inputs(lens, 2, dv, 0, with_state)
    layout = ChunkLayout(lens, torch.device(DEV))
    o, fin = fused_gated_delta_rule(q.to(DEV), k.to(DEV), v.to(DEV), gl.to(DEV), beta.to(DEV), layout,
                                    initial_state=s0.to(DEV) if s0 is not None else None)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    ref, fin_ref = naive_gated_delta_rule(q.float(), k.float(), v.float(), gl, beta, lens, initial_state=s0)
    assert rel_err(o.cpu(), ref) < 2e-2
    assert rel_err(fin.cpu(), fin_ref) < 2e-2


@pytest.mark.parametrize("lens,dv,with_state", [((150, 70, 300), 128, True), ((384, 128), 256, False)])
def test_fused_backward_matches_fp32_chunk_autograd(lens, dv, with_state):
    from prism_cp_b200.ops._lib import check_status
    from prism_cp_b200.ops.gdn import ChunkLayout, chunk_gated_delta_rule, fused_gated_delta_rule
    q, k, v, gl, beta, s0 = _inputs(lens, 2, dv, 1, with_state)
    gen = torch.Generator().manual_seed(7)
    T = sum(lens)
    w_o = torch.randn(T, 2, dv, generator=gen)
    w_f = torch.randn(len(lens), 2, 128, dv, generator=gen)

    def run(dev, fused):
        base = [q, k, v, gl, beta] + ([s0] if s0 is not None else [])
        ts = [b.detach().clone().to(dev) for b in base]
        if not fused:
            ts = [t.float() for t in ts]
        for t in ts:
            t.requires_grad_(True)
        layout = ChunkLayout(lens, torch.device(dev))
        init = ts[5] if s0 is not None else None
        fn = fused_gated_delta_rule if fused else chunk_gated_delta_rule
        o, fin = fn(*ts[:5], layout, initial_state=init)
        loss = (o.double() * w_o.to(dev).double()).sum() + (fin.double() * w_f.to(dev).double()).sum()
        loss.backward()
        return o.detach().cpu().double(), [t.grad.detach().cpu().double() for t in ts]

    o_ref, g_ref = run("cpu", False)
    o_gpu, g_gpu = run(DEV, True)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    assert rel_err(o_gpu, o_ref) < 2e-2
    names = ["q", "k", "v", "g", "beta", "s0"]
    for name, a, b in zip(names, g_gpu, g_ref):
        err = rel_err(a, b)
        assert err < 4e-2, f"d{name}: rel err {err}"


@pytest.mark.parametrize("module", ["gdn", "gqa", "mlp"])
def test_module_bench_gates_and_records(module, tmp_path):
    import json
    from prism_cp_b200.runtime import module_bench
    out = tmp_path / f"{module}.json"
    assert module_bench.main(["--module", module, "--cases", "4096,2x2048", "--output", str(out),
                              "--warmup", "1", "--iterations", "2"]) == 0
    doc = json.loads(out.read_text())
    assert {"repeat", "packed", "reference"} <= set(doc["gates"])
    assert len(doc["records"]) == 2 and all(r["fb_ms"] > 0 for r in doc["records"])


@pytest.mark.parametrize("lens,dv", [((150, 70, 300), 128), ((384, 128, 64), 256)])
def test_tensor_core_local_backward_matches_cuda_core_kernel(lens, dv):
    """The tcgen05 chunk-local backward and the CUDA-core one compute the same gradients
    (bf16 operands on the tensor cores: agreement to 2e-2 relative)."""
    from prism_cp_b200.ops._lib import check_status, lib
    from prism_cp_b200.ops.gdn import ChunkLayout, fused_gated_delta_rule
    q, k, v, gl, beta, _ = _inputs(lens, 3, dv, 5, False)
    w = torch.randn(sum(lens), 3, dv, generator=torch.Generator().manual_seed(3)).to(DEV)
    grads = {}
    for tc in (1, 0):
        lib().gdn_local_tc_enabled(tc)
        ts = [t.detach().clone().to(DEV).requires_grad_(True) for t in (q, k, v, gl, beta)]
        o, _ = fused_gated_delta_rule(*ts, ChunkLayout(lens, torch.device(DEV)))
        (o.float() * w).sum().backward()
        grads[tc] = [t.grad.float().cpu() for t in ts]
    lib().gdn_local_tc_enabled(1)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    for name, a, b in zip(("q", "k", "v", "g", "beta"), grads[1], grads[0]):
        assert torch.isfinite(a).all(), name
        assert rel_err(a, b) < 2e-2, f"d{name}: {rel_err(a, b)}"


@pytest.mark.parametrize("lens", [(1024,), (576, 448)])
def test_fused_affine_rule_matches_two_separate_passes(lens):
    """One prep for the zero-start pass and the identity pass of the first segment (dv contractions
    summed before one local backward) gives the outputs and gradients of the two separate passes."""
    from prism_cp_b200.ops.gdn import ChunkLayout, fused_affine_delta_rule, fused_gated_delta_rule
    dev = torch.device(DEV, torch.cuda.current_device())
    q, k, v, g, beta, _ = (t.to(dev) if t is not None else None for t in _inputs(lens, 4, 256, 7, False))
    layout, first = ChunkLayout(lens, dev), ChunkLayout(lens[:1], dev)
    n0, H, DK = lens[0], q.shape[1], q.shape[2]
    gen = torch.Generator(device=dev).manual_seed(3)
    w_o = torch.randn(sum(lens), H, 256, device=dev, generator=gen)
    w_L = torch.randn(n0, H, DK, device=dev, generator=gen)
    w_S = torch.randn(len(lens), H, DK, 256, device=dev, generator=gen)
    w_M = torch.randn(H, DK, DK, device=dev, generator=gen)

    def run(fused):
        ins = [t.detach().clone().requires_grad_(True) for t in (q, k, v, g, beta)]
        if fused:
            o, S, L, M = fused_affine_delta_rule(*ins, layout, first)
        else:
            o, S = fused_gated_delta_rule(*ins, layout)
            eye = torch.eye(DK, device=dev).expand(1, H, DK, DK).contiguous()
            L, Mf = fused_gated_delta_rule(ins[0][:n0], ins[1][:n0], torch.zeros_like(ins[0][:n0]), ins[3][:n0],
                                           ins[4][:n0], first, initial_state=eye)
            M = Mf[0]
        loss = (o.float() * w_o).sum() + (L.float() * w_L).sum() + (S * w_S).sum() + (M * w_M).sum()
        loss.backward()
        torch.cuda.synchronize()
        return [o.float(), L.float(), S, M] + [t.grad.float() for t in ins]

    a, b = run(True), run(False)
    names = ["o", "L", "S", "M", "dq", "dk", "dv", "dg", "dbeta"]
    for name, x, y in zip(names, a, b):
        err = ((x - y).norm() / y.norm().clamp_min(1e-6)).item()
        assert err < 1e-2, (name, err)
