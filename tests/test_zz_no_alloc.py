"""The allocation-free RMSNorm backward, called through its exported C symbol.

``prism_rmsnorm_bwd_noalloc`` exists for callers that cannot allocate device
memory themselves (no caching allocator, or allocation forbidden mid-step);
its working memory is a fixed array inside the library. This test calls it the
way such a caller would - by symbol, with raw pointers and a stream - and
checks consecutive calls (each on different data and sizes, so stale scratch
contents would show) against the regular PyTorch-facing entry point and an
fp32 PyTorch oracle.
The file is named so that pytest collects it after every other test.
"""

import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _library():
    import prism_cp_b200
    import prism_cp_b200._C  # noqa: F401  (loads the library into the process)
    path = glob.glob(os.path.join(os.path.dirname(prism_cp_b200.__file__), "_C*.so"))[0]
    lib = ctypes.CDLL(path)
    fn = lib.prism_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    msg = lib.prism_noalloc_error_string
    msg.restype = ctypes.c_char_p
    msg.argtypes = [ctypes.c_int]
    return fn, msg


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _case(rows, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, n, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(rows, n, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    return x, dy, w, rstd


def _oracle(x, dy, w, rstd):
    """fp32 PyTorch RMSNorm backward: dx and dw of y = x * rstd * w."""
    xf, dyf, wf = x.float(), dy.float(), w.float()
    xhat = xf * rstd[:, None]
    g = dyf * wf
    dx = rstd[:, None] * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    return dx, (dyf * xhat).sum(0)


# (rows, n): the last case has n at the 8192 maximum and enough rows that the number of
# partial-sum blocks is set by the scratch capacity (2^20 floats / 8192 = 128 blocks),
# not by the SM count or the row count
CASES = ((3000, 2048), (1500, 4096), (9000, 8192))


def test_noalloc_rmsnorm_backward_matches_regular_entry_point():
    from prism_cp_b200.ops._lib import lib
    fn, msg = _library()
    stream = torch.cuda.current_stream()
    for call, (rows, n) in enumerate(CASES):
        x, dy, w, rstd = _case(rows, n, seed=call)
        dx_ref = torch.empty_like(x)
        dw_ref = lib().rownorm_bwd(dy, x, w, None, rstd, dx_ref, None, 1, n, 1.0 / n)
        dx = torch.empty_like(x)
        dw = torch.full((n,), float("nan"), device="cuda")
        code = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                  rows, n, stream.cuda_stream)
        assert code == 0, msg(code).decode()
        torch.cuda.synchronize()
        assert rel_err(dx, dx_ref) < 1e-2
        assert rel_err(dw, dw_ref) < 1e-2
        dx_f32, dw_f32 = _oracle(x, dy, w, rstd)
        assert rel_err(dx, dx_f32) < 1e-2
        assert rel_err(dw, dw_f32) < 1e-2


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn, msg = _library()
    x, dy, w, rstd = _case(64, 16384, seed=7)
    out = torch.empty_like(x)
    dw = torch.empty(16384, device="cuda")
    code = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), out.data_ptr(), dw.data_ptr(), 64, 16384,
              torch.cuda.current_stream().cuda_stream)
    assert code == 2 and b"8192" in msg(code)


def test_noalloc_rejects_misaligned_fp32_pointers():
    fn, msg = _library()
    x, dy, w, rstd = _case(64, 1024, seed=9)
    out = torch.empty_like(x)
    dw = torch.empty(1024 + 4, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # rstd and dw are read and written as fp32: a pointer that is not 4-byte aligned is refused
    # before anything is launched
    code = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr() + 2, out.data_ptr(), dw.data_ptr(), 64,
              1024, stream)
    assert code == 1, msg(code).decode()
    code = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), out.data_ptr(), dw.data_ptr() + 1, 64,
              1024, stream)
    assert code == 1, msg(code).decode()
