"""Production supervisor: one fresh launch generation per platform (re)start, auto-resume.

Per node (reference ``train_production.py:39-154``):

1. take an exclusive per-node ``flock`` (never two attempts on one checkpoint stream);
2. ``join_attempt``: node 0 writes a new generation id; every node acknowledges it with a fresh
   per-process token; node 0 writes the cohort once all nodes acknowledged the same
   generation; a node proceeds only when the cohort lists its token (stale receipts from an
   earlier process can never be accepted); a changed node count is rejected;
3. start the training launcher in its own process group, logging under the attempt directory;
4. watch: if the generation changes, a peer reports a non-zero exit, or a signal arrives,
   SIGTERM the child group, then SIGKILL after 30 s;
5. publish ``exit_node_XXX.json``; when every node exited cleanly, node 0 writes
   ``complete.json`` (the finite dataset was consumed).
"""

from __future__ import annotations

import argparse
import fcntl
import json
import os
import signal
import subprocess
import sys
import time
import uuid
from pathlib import Path

from ..train.catalog import durable_json
from ..utils.files import atomic_json, read_json


def join_attempt(root, node_rank, nodes, timeout=1800.0, interval=0.5):
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    token = uuid.uuid4().hex
    generation = uuid.uuid4().hex if node_rank == 0 else None
    if node_rank == 0:
        atomic_json(root / "current.json", dict(generation=generation, nodes=nodes))
    deadline = time.monotonic() + timeout
    acknowledged = None
    while time.monotonic() < deadline:
        current = read_json(root / "current.json")
        if current is not None:
            if current["nodes"] != nodes:
                raise ValueError("restart node topology changed")
            active = current["generation"]
            if node_rank == 0 and active != generation:
                raise RuntimeError("another controller replaced this launch generation")
            if active != acknowledged:
                atomic_json(root / f"ack_{node_rank:03d}.json", dict(generation=active, token=token))
                acknowledged = active
            cohort_path = root / "attempts" / active / "cohort.json"
            if node_rank == 0:
                peers = [read_json(root / f"ack_{i:03d}.json") for i in range(nodes)]
                if all(p and p["generation"] == active for p in peers):
                    atomic_json(cohort_path, dict(generation=active, members=[p["token"] for p in peers]))
            cohort = read_json(cohort_path)
            if cohort and cohort["members"][node_rank] == token:
                return active
        time.sleep(interval)
    raise TimeoutError("a platform restart did not start every node of the fixed-size job")


def supervise(command, attempt, coordination, generation, node_rank, nodes, env=None, cwd=None, poll=0.5,
              grace=30.0):
    """Run ``command`` in a new session; stop it on generation change / peer failure; return its exit code."""
    attempt = Path(attempt)
    with (attempt / f"node_{node_rank:03d}.log").open("a") as log:
        child = subprocess.Popen(command, stdout=log, stderr=subprocess.STDOUT, start_new_session=True, env=env,
                                 cwd=cwd)
        stopped = [False]

        def terminate(signum=None, frame=None):
            stopped[0] = True
            if child.poll() is None:
                try:
                    os.killpg(child.pid, signal.SIGTERM)
                except ProcessLookupError:
                    pass

        old = {sig: signal.signal(sig, terminate) for sig in (signal.SIGTERM, signal.SIGINT)}
        try:
            while child.poll() is None:
                current = read_json(Path(coordination) / "current.json")
                peers = [read_json(attempt / f"exit_node_{i:03d}.json") for i in range(nodes)]
                if stopped[0] or (current and current["generation"] != generation) or any(p and p["exit_code"] for p in peers):
                    terminate()
                    try:
                        child.wait(timeout=grace)
                    except subprocess.TimeoutExpired:
                        os.killpg(child.pid, signal.SIGKILL)
                    break
                time.sleep(poll)
            code = child.wait()
            if stopped[0] and code == 0:
                code = 143
        finally:
            for sig, handler in old.items():
                signal.signal(sig, handler)
    atomic_json(attempt / f"exit_node_{node_rank:03d}.json", dict(exit_code=code))
    return code


def finish(output, attempt, generation, node_rank, nodes, timeout=1800.0, interval=0.5):
    deadline = time.monotonic() + timeout
    while time.monotonic() < deadline:
        peers = [read_json(Path(attempt) / f"exit_node_{i:03d}.json") for i in range(nodes)]
        if any(p and p["exit_code"] for p in peers):
            return 1
        if all(p is not None for p in peers):
            if node_rank == 0:
                durable_json(Path(output) / "complete.json", dict(generation=generation, status="finite_dataset_complete"))
            return 0
        time.sleep(interval)
    raise TimeoutError("training exited but peer nodes did not complete")


def training_command(args, attempt):
    root = Path(__file__).resolve().parents[2]
    train = ["--config", str(args.config), "--output", str(Path(attempt) / "train"),
             "--checkpoint-dir", str(Path(args.output) / "checkpoints"), "--resume"]
    if args.steps:
        train += ["--steps", str(args.steps)]
    return [sys.executable, "-m", "cq_pretrain_b200.launch.launcher", "--nodes", str(args.nodes),
            "--node-rank", str(args.node_rank), "--nproc-per-node", str(args.nproc_per_node),
            "--rendezvous", str(Path(attempt) / "rendezvous"), "--", *train], root


def run(args):
    output = Path(args.output)
    output.mkdir(parents=True, exist_ok=True)
    coordination = output / "coordination"
    coordination.mkdir(exist_ok=True)
    with (coordination / f"node_{args.node_rank:03d}.lock").open("a") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
        if (output / "complete.json").exists():
            print(json.dumps(dict(status="already_complete", output=str(output))), flush=True)
            return 0
        generation = join_attempt(coordination, args.node_rank, args.nodes)
        attempt = output / "attempts" / generation
        attempt.mkdir(parents=True, exist_ok=True)
        command, cwd = training_command(args, attempt)
        atomic_json(attempt / f"launch_node_{args.node_rank:03d}.json", dict(command=command, generation=generation))
        print(json.dumps(dict(status="launching", generation=generation, command=command)), flush=True)
        code = supervise(command, attempt, coordination, generation, args.node_rank, args.nodes, dict(os.environ),
                         str(cwd))
        if code:
            return code if code > 0 else 128 - code
        return finish(output, attempt, generation, args.node_rank, args.nodes)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--output", required=True, type=Path)
    parser.add_argument("--config", required=True, type=Path)
    parser.add_argument("--nodes", type=int, default=int(os.environ.get("PET_NNODES", "1")))
    parser.add_argument("--node-rank", type=int, default=int(os.environ.get("PET_NODE_RANK", "0")))
    parser.add_argument("--nproc-per-node", type=int, default=8)
    parser.add_argument("--steps", type=int, default=0)
    raise SystemExit(run(parser.parse_args(argv)))


if __name__ == "__main__":
    main()
