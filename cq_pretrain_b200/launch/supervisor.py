"""Production supervisor: one fresh launch generation per platform (re)start, auto-resume.

Per node (behaviour of the reference ``train_production.py:39-154``):

1. take an exclusive per-node ``flock`` (never two attempts on one checkpoint stream);
2. ``join_attempt`` agrees on a launch generation (protocol below);
3. start the training launcher in its own process group, logging under the attempt directory;
4. watch: if the generation changes, a peer reports a non-zero exit, or a signal arrives,
   SIGTERM the child group, then SIGKILL after 30 s;
5. publish ``exit_node_XXX.json``; when every node exited cleanly, node 0 writes
   ``complete.json`` (the finite dataset was consumed).

Generation protocol (files under the coordination directory):

* ``LATEST`` (JSON ``{generation, nodes}``): node 0 points it at a new random generation id each
  time it starts; a changed node count is refused by every node;
* ``generations/<id>/members/<rank>.json``: each node registers once per generation with a fresh
  per-process token, by exclusive create (a second registration of the same node fails; a
  sealed generation takes no registrations, it belongs to an earlier attempt);
* ``generations/<id>/sealed.json``: node 0 seals the generation with every member's token once
  all nodes registered. A node proceeds when the sealed list holds its own token, so a process
  that registered in an older generation can never pass for a member of the current one; a node
  that sees ``LATEST`` move on re-registers in the newer generation, and node 0 stops if another
  controller replaced its generation.
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

from ..utils.files import atomic_json, read_json


def current_generation(root):
    """``(generation, nodes)`` that ``LATEST`` names, or ``(None, None)`` before node 0 wrote it."""
    latest = read_json(Path(root) / "LATEST")
    return (latest["generation"], latest["nodes"]) if latest else (None, None)


def _register(root, generation, node_rank, token):
    members = Path(root) / "generations" / generation / "members"
    members.mkdir(parents=True, exist_ok=True)
    path = members / f"{node_rank:03d}.json"
    try:
        fd = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o644)
    except FileExistsError:
        raise RuntimeError(f"node {node_rank} is already registered in generation {generation} "
                           "by another process") from None
    with os.fdopen(fd, "w") as handle:
        json.dump(dict(token=token, pid=os.getpid()), handle)
    return path


def _seal_if_complete(root, generation, nodes):
    gen = Path(root) / "generations" / generation
    if (gen / "sealed.json").exists():
        return
    members = [read_json(gen / "members" / f"{r:03d}.json") for r in range(nodes)]
    if all(m is not None for m in members):
        atomic_json(gen / "sealed.json", dict(generation=generation, members=[m["token"] for m in members]))


def join_attempt(root, node_rank, nodes, timeout=1800.0, interval=0.5):
    """Block until every node joined one launch generation; returns its id."""
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    token = uuid.uuid4().hex
    mine = None
    if node_rank == 0:
        mine = uuid.uuid4().hex
        atomic_json(root / "LATEST", dict(generation=mine, nodes=nodes))
    registered = None
    give_up = time.monotonic() + timeout
    while time.monotonic() < give_up:
        generation, planned = current_generation(root)
        if generation is not None:
            if planned != nodes:
                raise ValueError(f"the job was planned for {planned} nodes, this node expects {nodes}")
            if mine is not None and generation != mine:
                raise RuntimeError("another controller started a newer launch generation")
            sealed_path = root / "generations" / generation / "sealed.json"
            if generation != registered and not sealed_path.exists():
                # a sealed generation belongs to an earlier attempt: wait for node 0 to start a new one
                _register(root, generation, node_rank, token)
                registered = generation
            if node_rank == 0:
                _seal_if_complete(root, generation, nodes)
            sealed = read_json(sealed_path)
            if sealed is not None and sealed["members"][node_rank] == token:
                return generation
        time.sleep(interval)
    raise TimeoutError(f"not every node of the {nodes}-node job joined a launch generation within {timeout:.0f} s")


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
                latest, _ = current_generation(coordination)
                peers = [read_json(attempt / f"exit_node_{i:03d}.json") for i in range(nodes)]
                if stopped[0] or (latest is not None and latest != generation) or any(p and p["exit_code"] for p in peers):
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
                atomic_json(Path(output) / "complete.json", dict(generation=generation, status="finite_dataset_complete"),
                            durable=True)
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
