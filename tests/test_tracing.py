"""Tracing hooks: NVTX ranges are free when disabled, the profiler window follows its steps."""

import torch

from prism_cp_b200.utils import tracing


def test_nvtx_disabled_is_a_null_context():
    tracing.enable_nvtx(False)
    with tracing.nvtx("layer 0"):
        x = 1
    assert x == 1 and not tracing.nvtx_enabled()


def test_nvtx_enabled_without_cuda_is_harmless():
    tracing.enable_nvtx(True)
    try:
        with tracing.nvtx("microbatch 0 forward"):
            pass
    finally:
        tracing.enable_nvtx(False)


def test_profile_window_inactive_off_rank_and_without_cuda():
    w = tracing.ProfileWindow(2, 3, ranks=[1], rank=0)
    assert not w.active
    for step in range(1, 5):
        w.before(step)
        w.after(step)
    assert not w.running
    w0 = tracing.ProfileWindow(2, 3, ranks=[0], rank=0)
    assert w0.active == torch.cuda.is_available()


def test_profile_window_rejects_inverted_range():
    import pytest
    with pytest.raises(ValueError):
        tracing.ProfileWindow(4, 3)


def test_launcher_accepts_profile_flags(tmp_path):
    from prism_cp_b200.launcher import train
    rc = train.main(["--device", "cpu", "--num-layers", "4", "--hidden-size", "256", "--ffn-hidden-size", "512",
                     "--vocab-size", "4096", "--num-attention-heads", "4", "--num-query-groups", "2",
                     "--kv-channels", "64", "--linear-num-key-heads", "4", "--linear-num-value-heads", "4",
                     "--linear-key-head-dim", "64", "--linear-value-head-dim", "64", "--global-batch-size", "2",
                     "--seq-length", "256", "--max-seqlen-per-dp-cp-rank", "512", "--train-iters", "2",
                     "--profile", "--profile-step-start", "1", "--profile-step-end", "2", "--nvtx-ranges"])
    tracing.enable_nvtx(False)
    assert rc == 0


def test_watchdog_reports_a_stall(capsys):
    import io
    import time
    from prism_cp_b200.utils.watchdog import StallWatchdog
    buf = io.StringIO()
    wd = StallWatchdog(1.0, stream=buf)
    try:
        wd.beat("layer 0 forward done")
        time.sleep(2.6)
        assert "no progress" in buf.getvalue() and "layer 0 forward done" in buf.getvalue()
        wd.beat("layer 1 forward done")
        assert not wd.reported
    finally:
        wd.close()


def test_timeline_summary_separates_hidden_and_exposed_communication():
    # compute 0..10 ms, NCCL 5..15 ms (5 ms hidden, 5 exposed), P2P 20..22 ms (exposed), idle 15..20
    kernels = [("prism::gemm::gemm_kernel", 0.0, 10000.0), ("ncclDevKernel_AllGather", 5000.0, 15000.0),
               ("prism::symm::gather_rows_kernel", 20000.0, 22000.0)]
    s = tracing.timeline_summary(kernels, 22.0)
    assert abs(s["span_ms"] - 22.0) < 1e-9 and abs(s["busy_ms"] - 17.0) < 1e-9
    assert abs(s["exposed_comm_ms"] - 7.0) < 1e-9 and abs(s["idle_ms"] - 5.0) < 1e-9
    assert s["categories"] == {"gemm": 10.0, "nccl": 10.0, "p2p": 2.0}
    assert tracing.categorize("void prism::attnb::attn_bwd_kv_kernel<prism::NoPeers>") == "attention"
    assert tracing.categorize("prism::gdnc::gdn_bwd_local_kernel") == "gdn"
    text = tracing.format_breakdown([dict(s, top=[("gemm", 10.0)])],
                                    dict(model="m", seqs=1, seq_len=8, world=1, impl="ring", plan="cp1", workload="fixed"))
    assert "| 0 | 22.0 | 17.0 | 5.0 | 7.0 |" in text
