"""The allocation-free RMSNorm backward, called through its exported C symbol.

``prism_rmsnorm_bwd_noalloc`` exists for callers that cannot allocate device
memory themselves (no caching allocator, or allocation forbidden mid-step);
its working memory is a fixed array inside the library. This test calls it the
way such a caller would - by symbol, with raw pointers and a stream - and
checks two consecutive calls (the second one on different data, so stale
scratch contents would show) against the regular PyTorch-facing entry point.
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


def test_noalloc_rmsnorm_backward_matches_regular_entry_point():
    from prism_cp_b200.ops._lib import lib
    fn, msg = _library()
    stream = torch.cuda.current_stream()
    for call, (rows, n) in enumerate(((3000, 2048), (1500, 4096))):
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


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn, msg = _library()
    x, dy, w, rstd = _case(64, 16384, seed=7)
    out = torch.empty_like(x)
    dw = torch.empty(16384, device="cuda")
    code = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), out.data_ptr(), dw.data_ptr(), 64, 16384,
              torch.cuda.current_stream().cuda_stream)
    assert code == 2 and b"8192" in msg(code)
