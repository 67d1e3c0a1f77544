"""Process groups for tensor (TP) and data (DP) parallelism over ``torch.distributed``.

One process per GPU; backend ``nccl`` on CUDA and ``gloo`` for CPU tests (reference
``distributed/megatron.py:53-91``, which used HCCL + Megatron ``parallel_state``). Ranks are laid
out TP-major: ranks ``[i*tp, (i+1)*tp)`` form TP group ``i`` (consecutive GPUs share an NVLink
domain either way on a single NVSwitch box); DP groups stride by ``tp``.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    world: int = 1
    rank: int = 0
    tp: int = 1
    tp_rank: int = 0
    dp: int = 1
    dp_rank: int = 0
    tp_group: object = None
    dp_group: object = None
    tp_ranks: tuple = (0,)
    dp_ranks: tuple = (0,)
    device: torch.device = torch.device("cpu")
    backend: str = "none"


_STATE = ParallelState()


def state() -> ParallelState:
    return _STATE


def tp_size() -> int:
    return _STATE.tp


def tp_rank() -> int:
    return _STATE.tp_rank


def dp_size() -> int:
    return _STATE.dp


def dp_rank() -> int:
    return _STATE.dp_rank


def initialize(tp: int = 1, backend: str | None = None, timeout_s: float = 600.0, device: str | None = None):
    """Initialise the default process group (if needed) and the TP/DP subgroups."""
    global _STATE
    if not dist.is_initialized():
        if "RANK" not in os.environ:
            _STATE = ParallelState(tp=1, device=torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu")))
            if tp != 1:
                raise ValueError("TP > 1 needs a distributed launch")
            if _STATE.device.type == "cuda":
                torch.cuda.set_device(0)
            return _STATE
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() and device != "cpu" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else None)
    backend = dist.get_backend()
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % tp:
        raise ValueError(f"world size {world} is not divisible by TP={tp}")
    dp = world // tp
    tp_group = dp_group = None
    my_tp = my_dp = None
    for i in range(dp):
        ranks = tuple(range(i * tp, (i + 1) * tp))
        group = dist.new_group(list(ranks))
        if rank in ranks:
            tp_group, my_tp = group, ranks
    for j in range(tp):
        ranks = tuple(range(j, world, tp))
        group = dist.new_group(list(ranks))
        if rank in ranks:
            dp_group, my_dp = group, ranks
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    _STATE = ParallelState(world, rank, tp, rank % tp, dp, rank // tp, tp_group, dp_group, my_tp, my_dp, dev, backend)
    return _STATE


def destroy():
    global _STATE
    if dist.is_initialized():
        dist.destroy_process_group()
    _STATE = ParallelState()


def set_state_for_tests(st: ParallelState):
    global _STATE
    _STATE = st
