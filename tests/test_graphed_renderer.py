"""CUDA-graphed renderer chunk against the same chunked backward run eagerly."""

import copy

import pytest
import torch


@pytest.mark.gpu
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


@pytest.mark.parametrize("env,tp,device,want", [
    ({}, 1, "cuda", True), ({}, 2, "cuda", True), ({"CQB_GRAPHS_TP": "0"}, 2, "cuda", False),
    ({"CQB_GRAPHS_TP": "0"}, 1, "cuda", True), ({"CQB_GRAPHS": "0"}, 1, "cuda", False), ({}, 1, "cpu", False)])
def test_graph_gating(monkeypatch, env, tp, device, want):
    """Which configurations replay the DiT chunk as a graph (no GPU needed: only the decision)."""
    from cq_pretrain_b200.config import tiny_config
    from cq_pretrain_b200.train.graphed import graphs_enabled
    for key in ("CQB_GRAPHS", "CQB_GRAPHS_TP"):
        monkeypatch.delenv(key, raising=False)
    for key, value in env.items():
        monkeypatch.setenv(key, value)
    cfg = tiny_config()
    assert graphs_enabled(cfg, device, tp) is want
    cfg.checkpoint_dit_layers = 2     # recomputed DiT blocks stay eager
    assert graphs_enabled(cfg, device, tp) is False


class _Optimizer:
    def __init__(self):
        self.waits = 0

    def wait_params(self):
        self.waits += 1


def test_graph_runner_waits_for_parameter_gathers_first():
    """Before any capture or replay the runner makes the stream wait for pending DP parameter
    all-gathers (their forward hooks must not wait inside a capture)."""
    from cq_pretrain_b200.train.graphed import RendererGraphs
    opt = _Optimizer()
    graphs = RendererGraphs(opt)       # the first sighting of a geometry runs eagerly (no CUDA needed)

    class Model:
        def renderer(self, leaf, bound):
            return (leaf * 2).sum()

    leaf = torch.ones(3, requires_grad=True)
    loss, grad = graphs.run(Model(), leaf, None, 1.0)
    assert opt.waits == 1 and float(loss) == 6.0 and torch.equal(grad, torch.full((3,), 2.0))
