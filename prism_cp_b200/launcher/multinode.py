"""Multi-node launcher: one process group per node, first failure stops the job.

``launch(hosts, command, output=...)`` starts ``command`` once per host with
``NODE_RANK``, ``NNODES``, ``MASTER_ADDR`` (the first host) and
``MASTER_PORT`` set, each in its own session (``setsid``) so the launcher can
stop exactly the processes it started. It polls all nodes; the first node that
exits non-zero, or the overall timeout, ends the job: every other node's
process group gets SIGTERM and, after a grace period, SIGKILL. The job writes
``launch.json`` (hosts, command, start time, pids) before starting and
``result.json`` (per-node exit codes, status, wall time) at the end. Same
behaviour as the reference's SSH launcher (scripts/torchrun_launcher.py:20-135:
setsid process groups, pidfiles, kill peers on the first failure, timeout).

Transports:

* ``ssh``: ``ssh -o BatchMode=yes <host> 'bash -lc <script>'``; the remote
  script records its process group in a pidfile and traps TERM to forward it
  to its children, so stopping the local ssh client and sending a remote
  ``kill -- -<pgid>`` both end the node's work;
* ``local``: the same script on this machine (single-box runs and tests).

Nothing is retried and an existing ``result.json`` is never overwritten.
"""

from __future__ import annotations

import argparse
import json
import os
import shlex
import signal
import subprocess
import sys
import time
import uuid
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class NodeProc:
    rank: int
    host: str
    proc: subprocess.Popen
    pidfile: str
    code: int | None = None
    killed: bool = False


@dataclass
class LaunchResult:
    status: str                       # "ok", "failed", "timeout"
    codes: list
    wall_s: float
    first_failure: int | None = None
    extra: dict = field(default_factory=dict)


def _remote_script(command: str, env: dict, pidfile: str, workdir: str | None) -> str:
    exports = " ".join(f"{k}={shlex.quote(str(v))}" for k, v in env.items())
    cd = f"cd {shlex.quote(workdir)} && " if workdir else ""
    # the node's own process group id goes to the pidfile; TERM is forwarded to the group
    return (f"echo $$ > {shlex.quote(pidfile)}; trap 'kill -TERM -- -$$ 2>/dev/null' TERM; "
            f"{cd}export {exports}; {command}")


def _spawn(rank: int, host: str, command: str, env: dict, transport: str, workdir: str | None,
           log_dir: Path) -> NodeProc:
    pidfile = f"/tmp/prism_launch_{uuid.uuid4().hex}_{rank}.pid"
    script = _remote_script(command, env, pidfile, workdir)
    if transport == "local":
        # start_new_session below makes the node's shell a session and process-group leader
        argv = ["bash", "-c", script]
    elif transport == "ssh":
        # remotely, setsid --wait gives the node its own group and returns the command's exit code
        argv = ["ssh", "-o", "BatchMode=yes", host, "bash -lc " + shlex.quote("setsid --wait bash -c " + shlex.quote(script))]
    else:
        raise ValueError(f"unknown transport {transport!r}")
    out = open(log_dir / f"node{rank}.log", "w")
    proc = subprocess.Popen(argv, stdout=out, stderr=subprocess.STDOUT, start_new_session=True)
    return NodeProc(rank, host, proc, pidfile)


def _stop(node: NodeProc, transport: str, grace_s: float) -> None:
    if node.proc.poll() is not None:
        return
    node.killed = True
    pgid = os.getpgid(node.proc.pid)
    if transport == "ssh":
        subprocess.run(["ssh", "-o", "BatchMode=yes", node.host,
                        f"kill -TERM -- -$(cat {shlex.quote(node.pidfile)}) 2>/dev/null"], timeout=30)
    try:
        os.killpg(pgid, signal.SIGTERM)
    except ProcessLookupError:
        return
    deadline = time.monotonic() + grace_s
    while time.monotonic() < deadline and node.proc.poll() is None:
        time.sleep(0.05)
    if node.proc.poll() is None:
        try:
            os.killpg(pgid, signal.SIGKILL)
        except ProcessLookupError:
            pass
        node.proc.wait()


def launch(hosts: list[str], command: str, output: str | Path, *, master_port: int = 29500, timeout_s: float = 3600,
           transport: str = "ssh", workdir: str | None = None, extra_env: dict | None = None, grace_s: float = 10.0,
           poll_s: float = 0.2) -> LaunchResult:
    out = Path(output)
    out.mkdir(parents=True, exist_ok=True)
    if (out / "result.json").exists():
        raise FileExistsError(f"{out / 'result.json'} exists; a launch never overwrites its result")
    master = hosts[0] if transport == "ssh" else "127.0.0.1"
    nodes: list[NodeProc] = []
    start = time.time()
    for rank, host in enumerate(hosts):
        env = {"NODE_RANK": rank, "NNODES": len(hosts), "MASTER_ADDR": master, "MASTER_PORT": master_port}
        env.update(extra_env or {})
        nodes.append(_spawn(rank, host, command, env, transport, workdir, out))
    (out / "launch.json").write_text(json.dumps({
        "hosts": hosts, "command": command, "transport": transport, "master_addr": master,
        "master_port": master_port, "start": start, "pids": [n.proc.pid for n in nodes],
        "pidfiles": [n.pidfile for n in nodes], "timeout_s": timeout_s}, indent=1))
    t0 = time.monotonic()
    status, first = "ok", None
    while True:
        running = 0
        for n in nodes:
            if n.code is None:
                c = n.proc.poll()
                if c is None:
                    running += 1
                else:
                    n.code = c
                    if c != 0 and first is None:
                        first = n.rank
        if first is not None:
            status = "failed"
            break
        if running == 0:
            break
        if time.monotonic() - t0 > timeout_s:
            status = "timeout"
            break
        time.sleep(poll_s)
    for n in nodes:
        _stop(n, transport, grace_s)
        if n.code is None:
            n.code = n.proc.returncode
        try:
            os.unlink(n.pidfile)
        except OSError:
            pass
    result = LaunchResult(status, [n.code for n in nodes], time.time() - start, first,
                          {"killed": [n.rank for n in nodes if n.killed]})
    (out / "result.json").write_text(json.dumps({
        "status": result.status, "codes": result.codes, "wall_s": result.wall_s,
        "first_failure": result.first_failure, "killed": result.extra["killed"]}, indent=1))
    return result


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="run one command per node; the first failure stops the job")
    ap.add_argument("--hosts", nargs="+", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--master-port", type=int, default=29500)
    ap.add_argument("--timeout", type=float, default=3600)
    ap.add_argument("--transport", choices=("ssh", "local"), default="ssh")
    ap.add_argument("--workdir", default=None)
    ap.add_argument("command", nargs=argparse.REMAINDER)
    args = ap.parse_args(argv)
    words = args.command[1:] if args.command[:1] == ["--"] else args.command
    cmd = " ".join(shlex.quote(c) for c in words)
    res = launch(args.hosts, cmd, args.output, master_port=args.master_port, timeout_s=args.timeout,
                 transport=args.transport, workdir=args.workdir)
    print(json.dumps({"status": res.status, "codes": res.codes}))
    return 0 if res.status == "ok" else 1


if __name__ == "__main__":
    sys.exit(main())
