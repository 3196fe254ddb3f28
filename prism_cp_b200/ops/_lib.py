"""Loader for the in-tree sm_100a kernel library ``prism_cp_b200._C``.

CUDA tensors always go through the compiled kernels; if the library is missing
on a machine with a GPU the first CUDA op raises instead of silently falling
back to PyTorch. CPU tensors use the plain PyTorch formulations in each op
module (fp32 oracle and the gloo/CPU plumbing path).
"""

from __future__ import annotations

import functools
import importlib
import os

import torch

# PRISM_KERNEL_DEBUG=1: load the bounds-checked build (``python -m prism_cp_b200.csrc.build --debug``)
DEBUG = os.environ.get("PRISM_KERNEL_DEBUG", "0") == "1"


class KernelLibraryMissing(RuntimeError):
    pass


@functools.lru_cache(maxsize=1)
def lib():
    name, flag = ("_C_debug", " --debug") if DEBUG else ("_C", "")
    try:
        return importlib.import_module(f"prism_cp_b200.{name}")
    except ImportError as error:  # pragma: no cover - exercised on GPU hosts only
        raise KernelLibraryMissing(
            f"prism_cp_b200.{name} is not built; run `python -m prism_cp_b200.csrc.build{flag}` "
            "(CUDA ops never fall back to PyTorch)") from error


_STATUS: dict[int, torch.Tensor] = {}


def status(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that bounded device waits write an error code into."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _STATUS.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _STATUS[index] = word
    return word


def check_status(device: torch.device) -> None:
    """Raise if any kernel on `device` recorded a timeout (synchronises)."""
    code = int(status(device).item())
    if code:
        status(device).zero_()
        if code == 6:
            raise RuntimeError("a prism kernel found an index outside its extent (debug build, code 6)")
        raise RuntimeError(f"device wait timed out in a prism kernel (code {code})")


def is_cuda(*tensors) -> bool:
    return any(t is not None and t.is_cuda for t in tensors)


def aligned_rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` if its rows are 16-byte aligned with unit inner stride, else a contiguous copy."""
    if t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(
            (t.stride(d) * t.element_size()) % 16 == 0 for d in range(t.dim() - 1)):
        return t
    return t.contiguous()


# ---------------------------------------------------------------- gradient-ready notifications
_GRAD_LISTENER = [None]


def set_grad_listener(fn) -> None:
    """Register ``fn(param)`` to be told when an op has accumulated into ``param.main_grad``."""
    _GRAD_LISTENER[0] = fn


def on_main_grad(param) -> None:
    fn = _GRAD_LISTENER[0]
    if fn is not None:
        fn(param)
