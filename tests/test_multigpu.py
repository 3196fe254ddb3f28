"""Multi-GPU paths (P2P reshard, ring attention, GDN CP) on 2+ GPUs via torchrun."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_multigpu_paths_match_single_gpu():
    n = min(torch.cuda.device_count(), 4)
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29517",
           os.path.join(here, "mgpu_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=660)
    assert res.returncode == 0 and "MGPU_OK" in res.stdout, res.stdout[-3000:] + res.stderr[-5000:]
