"""bench.py's command-line contract that needs no GPU: the reference arm's line and the options."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_unavailable_line_and_exits_zero():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference"], capture_output=True,
                         text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [x for x in res.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unavailable"]


def test_bench_options():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=300, cwd=ROOT)
    assert res.returncode == 0
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--workload", "--plan"):
        assert opt in res.stdout
