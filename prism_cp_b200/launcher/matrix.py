"""GPU run matrix: prepare arms from one input manifest, run them, summarise.

    python -m prism_cp_b200.launcher.matrix prepare   --manifest m.json --output runs --world 16 \\
        --arms fixed native joint --model hybrid-1.3b
    python -m prism_cp_b200.launcher.matrix run       --output runs --arm joint --hosts h0 h1 --nproc-per-node 8
    python -m prism_cp_b200.launcher.matrix summarize --output runs

``prepare`` validates the manifest and writes one directory per arm with the
launcher flags (``arm.json``): ``fixed`` (uniform CP = world), ``native`` (the
greedy dynamic-CP scheduler, its replay written for reference) and ``joint``
(the joint planner's frozen plan and replay, ``planner.cli search``). It never
overwrites an existing output.

``run`` starts ``worker`` on every host through the multi-node launcher
(first failure stops the job, no retry). ``worker`` is the per-node driver:
it validates the arm (manifest, replay rows against the pattern), lets node 0
write ``config.json``, ``numerical_contract.json`` and ``protocol.json`` while
the other nodes wait for them (bounded), sets the run environment and runs
``torchrun ... -m prism_cp_b200.launcher.train <flags>`` under ``timeout``,
with per-rank step records.

``summarize`` reads every arm's launch result and step records
(``runtime.records.summarize_records``) and writes ``comparison.json`` (status,
rank-max step seconds, tokens/s per arm) and ``supervision.json`` (the
contract checks per arm).

Reference: SD/random_batch_capacity_gpu.py:17-105 (prepare / run / worker /
summarize), SD/gpu_smoke.py:16-155 (per-node driver), without Megatron or a
sitecustomize hook: the launcher here is the training entry point itself.
"""

from __future__ import annotations

import argparse
import json
import os
import shlex
import subprocess
import sys
import time
from pathlib import Path

ARMS = ("fixed", "native", "joint")
PROTOCOL_WAIT_S = 120.0


def _model_flags(name: str) -> list[str]:
    from ..models.config import PRESETS
    c = PRESETS[name]()
    return ["--num-layers", str(c.num_layers), "--hidden-size", str(c.hidden_size),
            "--ffn-hidden-size", str(c.ffn_hidden_size), "--vocab-size", str(c.vocab_size),
            "--num-attention-heads", str(c.num_attention_heads), "--num-query-groups", str(c.num_query_groups),
            "--kv-channels", str(c.kv_channels), "--linear-num-key-heads", str(c.linear_num_key_heads),
            "--linear-num-value-heads", str(c.linear_num_key_heads),
            "--linear-key-head-dim", str(c.linear_key_head_dim),
            "--linear-value-head-dim", str(c.linear_value_head_dim),
            "--linear-attention-freq", str(c.linear_attention_freq)]


def prepare(manifest_path, output, world: int, arms=ARMS, model: str = "hybrid-1.3b", capacity: int = 32768,
            updates: int = 3, device: str = "cuda") -> dict:
    from ..planner.inputs import validate_manifest
    from ..planner.native import replay as native_replay
    out = Path(output)
    if out.exists():
        raise FileExistsError(f"{out} exists; prepare never overwrites a run matrix")
    manifest = json.loads(Path(manifest_path).read_text())
    validate_manifest(manifest)
    (out / "inputs").mkdir(parents=True)
    mpath = out / "inputs" / "manifest.json"
    mpath.write_text(json.dumps(manifest, indent=1))
    lengths = [s["length"] for s in manifest["samples"]]
    common = _model_flags(model) + ["--packet-manifest", str(mpath.resolve()), "--train-iters", str(updates),
                                    "--max-seqlen-per-dp-cp-rank", str(capacity), "--device", device]
    prepared = {}
    for arm in arms:
        d = out / "arms" / arm
        d.mkdir(parents=True)
        if arm == "fixed":
            flags = ["--sequence-packing-scheduler", "fixed", "--context-parallel-size", str(world)]
        elif arm == "native":
            rows = native_replay(list(enumerate(lengths)), world, capacity)
            (d / "native_replay.json").write_text(json.dumps(rows))
            flags = ["--sequence-packing-scheduler", "default_dynamic_cp"]
        elif arm == "joint":
            from ..planner import cli
            rc = cli.main(["search", "--manifest", str(mpath), "--output", str(d / "plan"), "--world", str(world),
                           "--model-config", model, "--updates", str(updates)])
            if rc != 0:
                raise RuntimeError(f"joint planner found no admissible plan for {manifest_path}")
            flags = ["--sequence-packing-scheduler", "joint", "--joint-replay", str((d / "plan" / "replay.json").resolve())]
        else:
            raise ValueError(f"unknown arm {arm!r}")
        spec = {"arm": arm, "world": world, "model": model, "flags": common + flags,
                "manifest": str(mpath.resolve()), "updates": updates}
        (d / "arm.json").write_text(json.dumps(spec, indent=1))
        prepared[arm] = spec
    (out / "matrix.json").write_text(json.dumps({"arms": list(arms), "world": world, "model": model,
                                                 "created": time.time()}, indent=1))
    return prepared


def _validate_arm(spec: dict) -> None:
    from ..models.config import PRESETS
    from ..planner.inputs import validate_manifest
    validate_manifest(json.loads(Path(spec["manifest"]).read_text()))
    pattern = PRESETS[spec["model"]]().pattern
    if set(pattern) - {"G", "*"} or "GGG*" * (len(pattern) // 4) != pattern:
        raise SystemExit(f"layer pattern {pattern!r} is not GGG* repeated")
    flags = spec["flags"]
    if "--joint-replay" in flags:
        from ..planner.joint.replay import validate_replay
        for row in json.loads(Path(flags[flags.index("--joint-replay") + 1]).read_text()):
            validate_replay(row, spec["world"], pattern)


def worker(output, arm: str, nproc_per_node: int, timeout_s: float = 3600, env_extra: dict | None = None) -> int:
    """Per-node driver (run on every node by ``run``)."""
    out = Path(output)
    spec = json.loads((out / "arms" / arm / "arm.json").read_text())
    _validate_arm(spec)
    node = int(os.environ.get("NODE_RANK", "0"))
    nnodes = int(os.environ.get("NNODES", "1"))
    run_dir = out / "arms" / arm / "run"
    protocol = run_dir / "protocol.json"
    if node == 0:
        run_dir.mkdir(parents=True, exist_ok=True)
        (run_dir / "config.json").write_text(json.dumps(spec, indent=1))
        (run_dir / "numerical_contract.json").write_text(json.dumps({"contract": "cp_bf16_v2"}, indent=1))
        protocol.write_text(json.dumps({"arm": arm, "nodes": nnodes, "nproc_per_node": nproc_per_node,
                                        "world": nnodes * nproc_per_node, "start": time.time()}, indent=1))
    else:
        t0 = time.monotonic()
        while not protocol.exists():
            if time.monotonic() - t0 > PROTOCOL_WAIT_S:
                print(f"node {node}: no protocol.json from node 0 after {PROTOCOL_WAIT_S:.0f} s", file=sys.stderr)
                return 3
            time.sleep(0.5)
    if nnodes * nproc_per_node != spec["world"]:
        print(f"arm {arm} was planned for {spec['world']} ranks, the job has {nnodes * nproc_per_node}",
              file=sys.stderr)
        return 4
    env = dict(os.environ)
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    env.update(env_extra or {})
    flags = spec["flags"] + ["--records", str(run_dir / "records")]
    if "--device" in flags and flags[flags.index("--device") + 1] == "cpu":
        flags += ["--distributed-backend", "gloo"]
    cmd = ["timeout", "--signal=TERM", "--kill-after=30s", f"{int(timeout_s)}s", sys.executable, "-m",
           "torch.distributed.run", f"--nnodes={nnodes}", f"--node-rank={node}",
           f"--nproc-per-node={nproc_per_node}", "--master-addr", env.get("MASTER_ADDR", "127.0.0.1"),
           "--master-port", env.get("MASTER_PORT", "29500"), "-m", "prism_cp_b200.launcher.train"] + flags
    return subprocess.run(cmd, env=env).returncode


def run(output, arm: str, hosts: list[str], nproc_per_node: int, transport: str = "ssh", timeout_s: float = 3600,
        master_port: int = 29500):
    from .multinode import launch
    out = Path(output).resolve()
    cmd = " ".join(shlex.quote(x) for x in [sys.executable, "-m", "prism_cp_b200.launcher.matrix", "worker",
                                             "--output", str(out), "--arm", arm,
                                             "--nproc-per-node", str(nproc_per_node), "--timeout", str(timeout_s)])
    return launch(hosts, cmd, out / "arms" / arm / "launch", master_port=master_port, timeout_s=timeout_s + 120,
                  transport=transport, workdir=os.getcwd())


def summarize(output) -> dict:
    from ..runtime.records import summarize_records
    out = Path(output)
    meta = json.loads((out / "matrix.json").read_text())
    manifest = json.loads((out / "inputs" / "manifest.json").read_text())
    comparison, supervision = {}, {}
    for arm in meta["arms"]:
        d = out / "arms" / arm
        spec = json.loads((d / "arm.json").read_text())
        launch_res = d / "launch" / "result.json"
        if not launch_res.exists():
            comparison[arm] = {"status": "not_run"}
            continue
        lr = json.loads(launch_res.read_text())
        steps = spec["updates"]
        rec = summarize_records(d / "run" / "records", manifest, steps, range(2, steps + 1) if steps > 1 else [1],
                                expected_batches=_expected_batches(d), world=meta["world"])
        status = rec["status"] if lr["status"] == "ok" else f"launch_{lr['status']}"
        entry = {"status": status, "launch": lr["status"]}
        if rec.get("mean_seconds"):
            entry["mean_rankmax_seconds"] = rec["mean_seconds"]
            entry["tokens_per_s"] = manifest["input_tokens"] / rec["mean_seconds"]
        comparison[arm] = entry
        supervision[arm] = {"checks": rec.get("checks"), "peak_GiB": rec.get("peak_GiB")}
    (out / "comparison.json").write_text(json.dumps(comparison, indent=1))
    (out / "supervision.json").write_text(json.dumps(supervision, indent=1))
    return comparison


def _expected_batches(arm_dir: Path):
    rec = arm_dir / "run" / "records"
    for f in sorted(rec.glob("steps_rank*.jsonl")):
        for line in f.read_text().splitlines():
            return json.loads(line)["execution_microbatches_per_update"]
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("prepare")
    p.add_argument("--manifest", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--world", type=int, required=True)
    p.add_argument("--arms", nargs="+", default=list(ARMS), choices=ARMS)
    p.add_argument("--model", default="hybrid-1.3b")
    p.add_argument("--capacity", type=int, default=32768)
    p.add_argument("--updates", type=int, default=3)
    p.add_argument("--device", default="cuda", choices=("cuda", "cpu"))
    r = sub.add_parser("run")
    r.add_argument("--output", required=True)
    r.add_argument("--arm", required=True)
    r.add_argument("--hosts", nargs="+", default=["localhost"])
    r.add_argument("--nproc-per-node", type=int, default=8)
    r.add_argument("--transport", choices=("ssh", "local"), default="ssh")
    r.add_argument("--timeout", type=float, default=3600)
    r.add_argument("--master-port", type=int, default=29500)
    w = sub.add_parser("worker")
    w.add_argument("--output", required=True)
    w.add_argument("--arm", required=True)
    w.add_argument("--nproc-per-node", type=int, default=8)
    w.add_argument("--timeout", type=float, default=3600)
    s = sub.add_parser("summarize")
    s.add_argument("--output", required=True)
    a = ap.parse_args(argv)
    if a.cmd == "prepare":
        prepare(a.manifest, a.output, a.world, a.arms, a.model, a.capacity, a.updates, a.device)
        return 0
    if a.cmd == "run":
        res = run(a.output, a.arm, a.hosts, a.nproc_per_node, a.transport, a.timeout, a.master_port)
        print(json.dumps({"status": res.status, "codes": res.codes}))
        return 0 if res.status == "ok" else 1
    if a.cmd == "worker":
        return worker(a.output, a.arm, a.nproc_per_node, a.timeout)
    print(json.dumps(summarize(a.output), indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
