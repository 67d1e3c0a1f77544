"""Fixed-size TP x DP launcher: rendezvous receipts, source agreement, then ``torchrun``.

Each node writes ``node{r}.json`` (hostname, address, interface, per-file source sha256, local
world size) into a fresh rendezvous directory, waits for every node, refuses to start unless all
nodes run identical sources with identical local world sizes, exports the NCCL/Gloo interface
and the master address of node 0, and ``exec``s ``torch.distributed.run`` on the training module
(reference ``launch_job.py:15-64`` + ``scripts/launch.sh``).
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import sys
from pathlib import Path

from ..utils.experiment import source_hashes
from ..utils.files import atomic_json, wait_files


def build_command(train_args, nodes, node_rank, nproc, master, port):
    return [sys.executable, "-m", "torch.distributed.run", f"--nnodes={nodes}", f"--node-rank={node_rank}",
            f"--nproc-per-node={nproc}", f"--master-addr={master}", f"--master-port={port}",
            "-m", os.environ.get("CQB_MODULE", "cq_pretrain_b200.train.loop"), *train_args]


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
    if args.nodes < 1 or not 0 <= args.node_rank < args.nodes or not train:
        raise ValueError("need a valid node topology and training arguments after --")
    master = os.environ.get("PET_MASTER_ADDR") or os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = os.environ.get("PET_MASTER_PORT") or os.environ.get("MASTER_PORT", "29500")
    if args.dry_run:
        print(json.dumps(dict(world=args.nodes * args.nproc_per_node, nodes=args.nodes, node_rank=args.node_rank,
                              command=build_command(train, args.nodes, args.node_rank, args.nproc_per_node, master, port),
                              rendezvous=str(args.rendezvous)), indent=2))
        return
    receipt = args.rendezvous / f"node{args.node_rank}.json"
    if receipt.exists():
        raise FileExistsError("use a new rendezvous directory for every launch/resume")
    sources = source_hashes()
    if args.nodes == 1:
        interface, address = "lo", "127.0.0.1"
    else:
        from ..utils.network import rendezvous_interface
        interface, addresses = rendezvous_interface(master)
        address = addresses[interface]
    atomic_json(receipt, dict(hostname=socket.gethostname(), ip=address, interface=interface,
                              source_sha256=sources, nproc=args.nproc_per_node))
    files = [args.rendezvous / f"node{n}.json" for n in range(args.nodes)]
    wait_files(files, 600)
    peers = [json.loads(p.read_text()) for p in files]
    if any(p["source_sha256"] != sources or p["nproc"] != args.nproc_per_node for p in peers):
        raise ValueError("all nodes must run the same sources and local world size")
    env = dict(os.environ, MASTER_ADDR=peers[0]["ip"], MASTER_PORT=port, GLOO_SOCKET_IFNAME=interface,
               NCCL_SOCKET_IFNAME=interface, TORCH_NCCL_ASYNC_ERROR_HANDLING="1",
               OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "4"))
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "GROUP_WORLD_SIZE"):
        env.pop(key, None)
    command = build_command(train, args.nodes, args.node_rank, args.nproc_per_node, peers[0]["ip"], port)
    os.execvpe(command[0], command, env)


if __name__ == "__main__":
    main()
