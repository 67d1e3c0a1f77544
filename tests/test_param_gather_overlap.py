"""The parameter all-gather overlapped with the next forward: every bucket a forward reads is
waited for by a forward pre-hook before the module that first reads it runs (CPU, fake works)."""

import torch

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.data.preparer import DevicePreparer
from cq_pretrain_b200.data.synthetic import synthetic_batch
from cq_pretrain_b200.parallel import state as ps
from cq_pretrain_b200.parallel.ddp import DistributedOptimizer
from cq_pretrain_b200.train.trainer import build_model


class FakeWork:
    def __init__(self, log, index):
        self.log, self.index = log, index

    def wait(self):
        self.log.append(self.index)


def test_forward_waits_for_every_bucket_once_in_forward_order():
    ps.initialize(1)
    cfg = tiny_config()
    model = build_model(cfg, torch.device("cpu"), dtype=torch.float32)
    opt = DistributedOptimizer(model, 1e-4, bucket_size=20_000, overlap_param_gather=True)
    assert len(opt.buckets) > 4
    log = []
    for b in opt.buckets:
        b.gather = (FakeWork(log, b.index), None)
    host, receipt = synthetic_batch(cfg, 512, seed=0, pad_multiple=8)
    batch = DevicePreparer(cfg, torch.device("cpu"), torch.float32)(host, receipt)
    with torch.no_grad():
        model(batch)
    # each bucket holding a parameter the forward reads was waited for exactly once
    assert len(log) == len(set(log))
    assert all(b.gather is None for b in opt.buckets if b.index in log)
    used = {opt.param_bucket[p].index for p in opt.param_bucket if p.requires_grad}
    missing = used - set(log)
    opt.wait_params()
    assert all(b.gather is None for b in opt.buckets)
    # buckets follow the backward order, so the forward reaches them (mostly) from the last one
    assert log[0] > log[-1], log
    assert not missing or len(missing) < len(used) // 4, missing
