"""In-tree build of the sm_100a kernel library.

``python -m prism_cp_b200.csrc.build`` compiles every ``.cu``/``.cpp`` file of
this directory for ``sm_100a`` only (explicit ``-gencode``; torch's own arch
list is emptied) into ``prism_cp_b200/_C*.so`` next to the package, so the
library travels with the source tree instead of living in a user cache.

``--debug`` builds the same sources with ``-DPRISM_BOUNDS_CHECK`` into
``prism_cp_b200/_C_debug*.so``: indices taken from host-built tables are
checked against their extents before the access and a bad one sets the
status word (error code 6) instead of faulting. ``PRISM_KERNEL_DEBUG=1``
makes ``ops._lib`` load that library.
"""

from __future__ import annotations

import glob
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PACKAGE = HERE.parent
BUILD_DIR = PACKAGE.parent / "_build" / "prism_C"
NAME = "_C"
DEBUG_NAME = "_C_debug"
DEBUG_FLAGS = ["-DPRISM_BOUNDS_CHECK"]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "--use_fast_math",
    "-Xptxas", "-v" if os.environ.get("PRISM_PTXAS_VERBOSE") else "-O3",
]


def sources() -> list[str]:
    files = sorted(glob.glob(str(HERE / "*.cu"))) + sorted(glob.glob(str(HERE / "*.cpp")))
    return files


def build(verbose: bool = False, debug: bool = False) -> Path:
    os.environ["TORCH_CUDA_ARCH_LIST"] = ""  # only the explicit -gencode above
    from torch.utils import cpp_extension

    name = DEBUG_NAME if debug else NAME
    build_dir = BUILD_DIR.parent / ("prism_C_debug" if debug else "prism_C")
    extra = DEBUG_FLAGS if debug else []
    build_dir.mkdir(parents=True, exist_ok=True)
    jobs = os.environ.get("MAX_JOBS") or str(max(1, os.cpu_count() or 1))
    os.environ["MAX_JOBS"] = jobs
    cpp_extension.load(
        name=name,
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"] + extra,
        extra_cuda_cflags=CUDA_FLAGS + extra,
        extra_include_paths=[str(HERE)],
        build_directory=str(build_dir),
        verbose=verbose,
        with_cuda=True,
        is_python_module=True,
    )
    built = sorted(build_dir.glob(f"{name}*.so"))
    if not built:
        raise RuntimeError("kernel library build produced no shared object")
    target = PACKAGE / built[0].name
    shutil.copy2(built[0], target)
    return target


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, debug="--debug" in sys.argv)
    print(path)
