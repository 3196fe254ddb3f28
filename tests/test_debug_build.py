"""The bounds-checked debug variant of the kernels (``python -m prism_cp_b200.csrc.build --debug``)."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "prism_cp_b200" / "csrc"

PROBE = r"""
#include "common.cuh"
// a gather through a host-built index table, checked the way the kernels check theirs
__global__ void probe(const int* table, int n_table, const float* src, int n_src, float* dst, int* status) {
  const int i = threadIdx.x;
  if (!PRISM_IN_BOUNDS(i, n_table, status)) return;
  const int j = table[i];
  if (PRISM_IN_BOUNDS(j, n_src, status)) dst[i] = src[j];
}
"""


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not installed")
@pytest.mark.parametrize("debug", [False, True])
def test_bounds_check_macro_compiles_for_sm100a(tmp_path, debug):
    from prism_cp_b200.csrc.build import CUDA_FLAGS, DEBUG_FLAGS
    src = tmp_path / "probe.cu"
    src.write_text(PROBE)
    flags = [f for f in CUDA_FLAGS if f not in ("-Xptxas", "-v", "-O3")] + (DEBUG_FLAGS if debug else [])
    out = subprocess.run(["nvcc", "-c", str(src), "-o", str(tmp_path / "probe.o"), f"-I{CSRC}"] + flags,
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr[-4000:]


def test_release_build_has_no_bounds_checks():
    """In the release build the checks are the constant true (no extra loads or branches); the
    kernels that index through host-built tables carry them."""
    text = (CSRC / "common.cuh").read_text()
    assert "#define PRISM_IN_BOUNDS(idx, extent, status) true" in text
    uses = {f: (CSRC / f).read_text().count("PRISM_IN_BOUNDS(") for f in
            ("symm.cu", "attention_fwd_sm100.cu", "attention_bwd_sm100.cu", "gdn_chunk.cu")}
    assert all(uses.values()) and sum(uses.values()) >= 8, uses
