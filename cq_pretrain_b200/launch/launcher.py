"""Fixed-size TP x DP launcher: rendezvous receipts, source agreement, then ``torchrun``.

Each node publishes a ``Receipt`` (hostname, address and interface toward node 0, sha256 of
every source file, processes per node) into a fresh rendezvous directory, collects every node's
receipt, and starts training only if all nodes run byte-identical sources with the same number of
processes; ``disagreements`` names each offending node and the files that differ. The launch
environment points NCCL and Gloo at the chosen interface and at node 0's address, and the process
``exec``s ``torch.distributed.run`` on the training module (behaviour of the reference
``launch_job.py:15-64`` and ``scripts/launch.sh``).
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import sys
import time
from dataclasses import asdict, dataclass
from pathlib import Path

from ..utils.experiment import source_hashes
from ..utils.files import wait_files

# variables torchrun sets per process: a parent's values must not leak into the children
_PER_PROCESS = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "GROUP_WORLD_SIZE")


@dataclass
class Receipt:
    hostname: str
    ip: str
    interface: str
    source_sha256: dict
    nproc: int


class Rendezvous:
    """One directory per launch: ``node{r}.json`` per node, created exclusively."""

    def __init__(self, directory, nodes, node_rank):
        if nodes < 1 or not 0 <= node_rank < nodes:
            raise ValueError(f"node rank {node_rank} is not valid for a {nodes}-node job")
        self.directory, self.nodes, self.node_rank = Path(directory), nodes, node_rank

    def path(self, rank):
        return self.directory / f"node{rank}.json"

    def publish(self, receipt: Receipt):
        self.directory.mkdir(parents=True, exist_ok=True)
        try:
            fd = os.open(self.path(self.node_rank), os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o644)
        except FileExistsError:
            raise FileExistsError(f"{self.directory} already holds a receipt of node {self.node_rank}: "
                                  "every launch or resume needs a new rendezvous directory") from None
        with os.fdopen(fd, "w") as handle:
            json.dump(asdict(receipt), handle)

    def collect(self, timeout=600.0):
        paths = [self.path(r) for r in range(self.nodes)]
        wait_files(paths, timeout)
        receipts = []
        for p in paths:
            for _ in range(50):     # a peer's exclusive-create file may still be being written
                try:
                    receipts.append(Receipt(**json.loads(p.read_text())))
                    break
                except ValueError:
                    time.sleep(0.1)
            else:
                raise ValueError(f"unreadable receipt {p}")
        return receipts


def disagreements(receipts, mine: Receipt):
    """Why the nodes may not start together (empty when they agree)."""
    problems = []
    for rank, other in enumerate(receipts):
        if other.nproc != mine.nproc:
            problems.append(f"node {rank} runs {other.nproc} processes, this node {mine.nproc}")
        if other.source_sha256 != mine.source_sha256:
            names = sorted(k for k in other.source_sha256.keys() | mine.source_sha256.keys()
                           if other.source_sha256.get(k) != mine.source_sha256.get(k))
            problems.append(f"node {rank} has different sources: {names[:6]}{' ...' if len(names) > 6 else ''}")
    return problems


def build_command(train_args, nodes, node_rank, nproc, master, port):
    return [sys.executable, "-m", "torch.distributed.run", f"--nnodes={nodes}", f"--node-rank={node_rank}",
            f"--nproc-per-node={nproc}", f"--master-addr={master}", f"--master-port={port}",
            "-m", os.environ.get("CQB_MODULE", "cq_pretrain_b200.train.loop"), *train_args]


def launch_environment(base, master_ip, port, interface):
    env = {k: v for k, v in base.items() if k not in _PER_PROCESS}
    env.update(MASTER_ADDR=master_ip, MASTER_PORT=str(port), GLOO_SOCKET_IFNAME=interface,
               NCCL_SOCKET_IFNAME=interface, TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    env.setdefault("OMP_NUM_THREADS", "4")
    return env


def _local_receipt(nodes, master, nproc):
    if nodes == 1:
        interface, ip = "lo", "127.0.0.1"
    else:
        from ..utils.network import rendezvous_interface
        interface, addresses = rendezvous_interface(master)
        ip = addresses[interface]
    return Receipt(socket.gethostname(), ip, interface, source_hashes(), nproc)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--rendezvous", required=True, type=Path, help="fresh shared directory for this launch")
    parser.add_argument("--nodes", type=int, default=int(os.environ.get("PET_NNODES", "1")))
    parser.add_argument("--node-rank", type=int, default=int(os.environ.get("PET_NODE_RANK", "0")))
    parser.add_argument("--nproc-per-node", type=int, default=8)
    parser.add_argument("--dry-run", action="store_true")
    parser.add_argument("training_args", nargs=argparse.REMAINDER)
    args = parser.parse_args(argv)
    train = args.training_args[1:] if args.training_args[:1] == ["--"] else args.training_args
    if not train:
        raise ValueError("pass the training arguments after --")
    rendezvous = Rendezvous(args.rendezvous, args.nodes, args.node_rank)
    master = os.environ.get("PET_MASTER_ADDR") or os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = os.environ.get("PET_MASTER_PORT") or os.environ.get("MASTER_PORT", "29500")
    if args.dry_run:
        print(json.dumps(dict(world=args.nodes * args.nproc_per_node, nodes=args.nodes, node_rank=args.node_rank,
                              command=build_command(train, args.nodes, args.node_rank, args.nproc_per_node, master,
                                                    port),
                              rendezvous=str(args.rendezvous)), indent=2))
        return
    mine = _local_receipt(args.nodes, master, args.nproc_per_node)
    rendezvous.publish(mine)
    receipts = rendezvous.collect()
    problems = disagreements(receipts, mine)
    if problems:
        raise ValueError("the nodes cannot start one job: " + "; ".join(problems))
    env = launch_environment(os.environ, receipts[0].ip, port, mine.interface)
    command = build_command(train, args.nodes, args.node_rank, args.nproc_per_node, receipts[0].ip, port)
    os.execvpe(command[0], command, env)


if __name__ == "__main__":
    main()
