"""Run matrix: prepare arms from a manifest, run them through the launcher on CPU ranks, summarise."""

import json

import pytest

from prism_cp_b200.launcher import matrix
from prism_cp_b200.planner.inputs import build_manifest


def test_prepare_run_summarize_cpu(tmp_path):
    manifest = build_manifest([384, 256, 128, 256], "tiny", 2, seed=5, vocab=4096)
    mpath = tmp_path / "m.json"
    mpath.write_text(json.dumps(manifest))
    out = tmp_path / "runs"
    arms = matrix.prepare(mpath, out, world=2, arms=("fixed", "native", "joint"), model="hybrid-tiny",
                          capacity=512, updates=2, device="cpu")
    assert set(arms) == {"fixed", "native", "joint"}
    # the joint planner plans the preset's own layers
    result = json.loads((out / "arms" / "joint" / "plan" / "result.json").read_text())
    assert result["plan"]["pattern"] == "GGG*"
    assert (out / "arms" / "native" / "native_replay.json").exists()
    with pytest.raises(FileExistsError):
        matrix.prepare(mpath, out, world=2, arms=("fixed",), model="hybrid-tiny", device="cpu")
    for i, arm in enumerate(("fixed", "native", "joint")):
        res = matrix.run(out, arm, ["localhost"], nproc_per_node=2, transport="local", timeout_s=240,
                         master_port=29650 + i)
        assert res.status == "ok", (out / "arms" / arm / "launch" / "node0.log").read_text()[-3000:]
        assert (out / "arms" / arm / "run" / "protocol.json").exists()
    comp = matrix.summarize(out)
    for arm in ("fixed", "native", "joint"):
        assert comp[arm]["launch"] == "ok"
        assert comp[arm]["status"] in ("complete", "actual_memory_guard_rejected"), comp
    sup = json.loads((out / "supervision.json").read_text())
    assert sup["fixed"]["checks"]["input_tokens"] and sup["native"]["checks"]["finite"]


def test_worker_rejects_a_world_mismatch(tmp_path, monkeypatch):
    manifest = build_manifest([256, 256], "tiny", 2, seed=1, vocab=4096)
    mpath = tmp_path / "m.json"
    mpath.write_text(json.dumps(manifest))
    out = tmp_path / "runs"
    matrix.prepare(mpath, out, world=2, arms=("fixed",), model="hybrid-tiny", capacity=512, updates=1, device="cpu")
    monkeypatch.setenv("NODE_RANK", "0")
    monkeypatch.setenv("NNODES", "1")
    assert matrix.worker(out, "fixed", nproc_per_node=4) == 4
