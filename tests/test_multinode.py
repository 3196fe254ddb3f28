"""Multi-node launcher on the local transport: success, first-failure stop, timeout, no overwrite."""

import json
import time

import pytest

from prism_cp_b200.launcher.multinode import launch


def test_all_nodes_succeed_and_see_their_rank(tmp_path):
    out = tmp_path / "ok"
    res = launch(["a", "b", "c"], 'echo "rank=$NODE_RANK of $NNODES at $MASTER_ADDR:$MASTER_PORT"', out,
                 transport="local", master_port=29611, timeout_s=30)
    assert res.status == "ok" and res.codes == [0, 0, 0]
    for r in range(3):
        assert f"rank={r} of 3 at 127.0.0.1:29611" in (out / f"node{r}.log").read_text()
    launch_meta = json.loads((out / "launch.json").read_text())
    assert launch_meta["hosts"] == ["a", "b", "c"] and len(launch_meta["pids"]) == 3
    assert json.loads((out / "result.json").read_text())["status"] == "ok"


def test_first_failure_stops_the_other_nodes(tmp_path):
    out = tmp_path / "fail"
    t0 = time.monotonic()
    cmd = 'if [ "$NODE_RANK" = 1 ]; then sleep 0.3; exit 3; else sleep 60; fi'
    res = launch(["a", "b"], cmd, out, transport="local", timeout_s=60, grace_s=2)
    assert res.status == "failed" and res.first_failure == 1
    assert res.codes[1] == 3 and res.codes[0] != 0
    assert time.monotonic() - t0 < 20
    assert json.loads((out / "result.json").read_text())["killed"] == [0]


def test_timeout_stops_every_node_and_never_overwrites(tmp_path):
    out = tmp_path / "slow"
    res = launch(["a", "b"], "sleep 60", out, transport="local", timeout_s=0.5, grace_s=2)
    assert res.status == "timeout" and all(c != 0 for c in res.codes)
    with pytest.raises(FileExistsError):
        launch(["a"], "true", out, transport="local")
