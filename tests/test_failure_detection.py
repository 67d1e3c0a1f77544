"""Failure detection without faulting anything.

* CPU (gloo): a rank that leaves between steps makes the survivor's next collective fail with
  an error within the process-group timeout instead of hanging.
* GPU: a flag wait that nothing satisfies expires after its bound (~2 s), records an error status
  that the host reads, and leaves the CUDA context usable.
"""

import os
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _leaver(rank, world, store, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)          # step 1: everyone present
    if rank == 1:
        os._exit(0)             # leaves between steps, with nothing in flight
    time.sleep(0.5)
    start = time.monotonic()
    try:
        dist.all_reduce(t)      # step 2: the peer is gone
        outcome = "completed"
    except Exception as error:  # noqa: BLE001 - any error is the detection we want
        outcome = type(error).__name__
    Path(out).write_text(f"{outcome} {time.monotonic() - start:.1f}")


def test_departed_rank_fails_next_collective():
    with tempfile.TemporaryDirectory() as tmp:
        out = Path(tmp) / "out"
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_leaver, args=(r, 2, str(Path(tmp) / "store"), str(out))) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(60)
            assert not p.is_alive()
        outcome, seconds = out.read_text().split()
    assert outcome != "completed" and float(seconds) < 30


@pytest.mark.gpu
def test_flag_wait_times_out_with_status():
    from cq_pretrain_b200.ops import _ext
    ops = _ext.ops()
    ops.comm_status_read(True)
    mine = torch.zeros(8, dtype=torch.int64, device="cuda")      # this rank's flag slots
    elsewhere = torch.zeros(8, dtype=torch.int64, device="cuda")  # stands in for a peer that never answers
    peers = torch.tensor([mine.data_ptr(), elsewhere.data_ptr()], dtype=torch.int64, device="cuda")
    start = time.monotonic()
    # rank 0 of 2: publishes epoch 3 to both "peers", then waits for slot 1 of its own area,
    # which no one ever sets -> the bounded wait expires
    ops.signal_wait(peers, mine.data_ptr(), 0, 2, 3, True)
    torch.cuda.synchronize()
    elapsed = time.monotonic() - start
    assert ops.comm_status_read(True) == 101          # 100 + the slot that never arrived
    assert 1.0 < elapsed < 30.0
    assert int(mine[0]) == 3 and int(elsewhere[0]) == 3
    # the context is still usable
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert torch.equal((x * 2).cpu(), torch.arange(0, 2048, 2, dtype=torch.float32))
    assert ops.comm_status_read(False) == 0
