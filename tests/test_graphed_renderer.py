"""CUDA-graphed renderer chunk against the same chunked backward run eagerly."""

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_graphed_renderer_matches_eager_over_steps():
    from cq_pretrain_b200.config import tiny_config
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.ops import _ext
    from cq_pretrain_b200.train.graphed import RendererGraphs
    from cq_pretrain_b200.train.trainer import Trainer
    cfg = tiny_config()
    host, receipt = synthetic_batch(cfg, 512, seed=4, pad_multiple=128)
    host = host.pin_memory()
    graphed = Trainer(copy.deepcopy(cfg), tp=1, lr=1e-3, ema_decay=0.999, device="cuda:0", seed=11)
    eager = Trainer(copy.deepcopy(cfg), tp=1, lr=1e-3, ema_decay=0.999, device="cuda:0", seed=11)
    assert graphed.renderer_graphs is not None
    eager.renderer_graphs = RendererGraphs(eager.optimizer, capture_after=10 ** 9)   # same schedule, never captured
    counts = []
    for step in range(4):   # eager sighting, capture + replay, then two plain replays
        item = (host, dict(receipt, serial=receipt["serial"] + step))   # new flow noise and times each step
        before = _ext.launches()
        a = graphed.train_step([item])
        torch.cuda.synchronize()
        counts.append(_ext.launches() - before)
        b = eager.train_step([item])
        assert abs(a["loss"] - b["loss"]) <= 1e-3 * abs(b["loss"]) + 1e-5, (step, a, b)
        assert abs(a["grad_norm"] - b["grad_norm"]) <= 1e-3 * b["grad_norm"] + 1e-6, (step, a, b)
    assert graphed.renderer_graphs.replays == 3 and eager.renderer_graphs.replays == 0
    assert len(set(counts)) == 1, counts     # replays count the extension kernels they run
    for (name, p), (_, q) in zip(graphed.model.named_parameters(), eager.model.named_parameters()):
        rel = (p.float() - q.float()).norm() / q.float().norm().clamp_min(1e-12)
        assert rel < 2e-3, (name, rel.item())
