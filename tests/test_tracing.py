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
