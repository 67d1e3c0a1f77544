"""Training invariants of the reference's test suite, on CPU (gloo ranks where several are needed).

* the chunked renderer backward gives the unchunked loss and every gradient (reference
  ``tests/test_wan_unified.py:84-109``);
* DP/GA loss scales make sparse image objectives a global average (``tests/test_i2t_loss_scaling.py``);
* TP=2 equals TP=1 for the whole tiny joint model (gloo);
* a DP rank without generation targets issues the same collective sequence as one with them
  (``tests/test_collective_order.py``);
* the EMA install/restore and the evaluation-snapshot round trip at world 4 (TP2 x DP2,
  ``tests/test_eval_snapshot.py:28-60``).
"""

import os
import tempfile
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cq_pretrain_b200.config import tiny_config


def _cfg(**kw):
    base = dict(layers=4, dit_layers=2, vocab_size=256, width=128, ffn=256, heads=4, kv_heads=2, head_dim=32,
                mrope_section=(2, 1, 1), linear_heads=2, linear_head_dim=32, dit_width=64, dit_heads=4, dit_ffn=128)
    base.update(kw)
    return tiny_config(**base)


def _prepared(cfg, tp=1, seed=3, dp_rank=0, dtype=torch.float32, **kw):
    from cq_pretrain_b200.data.preparer import DevicePreparer
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    host, receipt = synthetic_batch(cfg, 256, seed=seed + dp_rank, pad_multiple=8 * tp, **kw)
    return DevicePreparer(cfg, torch.device("cpu"), dtype)(host, receipt)


def _grads(model):
    return {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}


# ---- chunked renderer backward ------------------------------------------------------------------
def test_chunked_renderer_backward_matches_unchunked():
    from cq_pretrain_b200.parallel import state as ps
    from cq_pretrain_b200.train.loss import compose_losses
    from cq_pretrain_b200.train.renderer_schedule import backward_deferred_renderer
    from cq_pretrain_b200.train.trainer import build_model
    ps.initialize(1)
    cfg = _cfg(generation_microbatch_images=1)
    batch = _prepared(cfg)
    assert len(batch.generation.microbatches) >= 2, "the test needs several DiT chunks"
    results = []
    for chunked in (True, False):
        model = build_model(cfg, torch.device("cpu"), seed=7, dtype=torch.float32)
        out = model(batch, compute_image_loss=not chunked)
        losses = compose_losses(out, cfg, (1.0, 1.0))
        if chunked:
            losses = backward_deferred_renderer(model, batch, losses, 1.0, None, image_factor=cfg.image_weight)
        else:
            losses["loss"].backward()
        results.append((float(losses["loss"]), float(losses["image_loss"]), _grads(model)))
    (la, ia, ga), (lb, ib, gb) = results
    assert abs(la - lb) < 1e-5 * max(1.0, abs(lb)) and abs(ia - ib) < 1e-5 * max(1.0, abs(ib))
    assert ga.keys() == gb.keys() and len(ga) > 20
    for name in gb:
        torch.testing.assert_close(ga[name], gb[name], rtol=2e-4, atol=2e-6, msg=name)


# ---- DP / GA loss scales --------------------------------------------------------------------------
def test_sparse_image_objectives_average_globally():
    from cq_pretrain_b200.train.loss import scales_from_counts
    # (text targets, per-image regression targets) per pack; two replicas of two packs each, two packs
    # without generation targets: the renderer loss must be the mean over the 3 selected images
    packs = [[(3, [1.0, 3.0]), (5, [])], [(2, []), (4, [5.0])]]
    dp, total_text, total_images = 2, 14, 3
    actual = torch.tensor(0.7, requires_grad=True)
    total = actual * 0
    for replica in packs:
        for text, targets in replica:
            _, s_i = scales_from_counts(text, len(targets), total_text, total_images, dp)
            loss = (actual - torch.tensor(targets)).square().mean() if targets else actual * 0
            total = total + loss * s_i / dp
    total.backward()
    expected = torch.tensor(0.7, requires_grad=True)
    oracle = (expected - torch.tensor([1.0, 3.0, 5.0])).square().mean()
    oracle.backward()
    torch.testing.assert_close(total, oracle)
    torch.testing.assert_close(actual.grad, expected.grad)
    # no targets anywhere: the image scale is 0 and the text scale keeps its share
    assert scales_from_counts(7, 0, 14, 0, 2) == (1.0, 0.0)
    assert scales_from_counts(0, 0, 0, 0, 2) == (0.0, 0.0)


# ---- multi-rank (gloo) ----------------------------------------------------------------------------
def _init(rank, world, store):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)


def _spawn(fn, world, *args):
    mp.start_processes(fn, args=(world, *args), nprocs=world, start_method="spawn", join=True)


def _tp_worker(rank, world, store, reference, out):
    _init(rank, world, store)
    from cq_pretrain_b200.parallel import layers as PL
    from cq_pretrain_b200.parallel import state as ps
    from cq_pretrain_b200.train.reshard import reshard_state
    from cq_pretrain_b200.train.trainer import build_model
    st = ps.initialize(world, backend="gloo", device="cpu")
    ref = torch.load(reference)
    cfg = _cfg()
    model = build_model(cfg, torch.device("cpu"), seed=7, dtype=torch.float32).double()
    with torch.no_grad():
        model.load_state_dict(reshard_state([ref["state"]], model, st.tp, st.tp_rank), strict=True)
    batch = _prepared(cfg, tp=st.tp, dtype=torch.float64)
    out_ = model(batch)
    loss = out_["text_loss"] + out_["image_loss"]
    loss.backward()
    errors = {"text_loss": abs(float(out_["text_loss"]) - ref["text"]) / abs(ref["text"]),
              "image_loss": abs(float(out_["image_loss"]) - ref["image"]) / abs(ref["image"])}
    params = dict(model.named_parameters())
    for name, p in params.items():
        if p.grad is None:
            continue
        g = p.grad.detach().clone()
        if not getattr(p, "tensor_model_parallel", False) and not getattr(p, "tp_duplicate", False):
            dist.all_reduce(g, group=st.tp_group)          # replicated parameters: partial gradients
        want = PL.checkpoint_shard(ref["grads"][name], p)
        errors[name] = float((g - want).norm() / want.norm().clamp_min(1e-12))
    torch.save(errors, f"{out}.{rank}")
    dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_joint_model_tp2_matches_tp1():
    from cq_pretrain_b200.parallel import state as ps
    from cq_pretrain_b200.train.trainer import build_model
    ps.initialize(1)
    cfg = _cfg()
    # float64 end to end: some decay-parameter gradients are ~1e-7 and dominated by cancellation
    model = build_model(cfg, torch.device("cpu"), seed=7, dtype=torch.float32).double()
    batch = _prepared(cfg, tp=2, dtype=torch.float64)  # the same padded pack as the TP2 ranks see
    out = model(batch)
    (out["text_loss"] + out["image_loss"]).backward()
    with tempfile.TemporaryDirectory() as tmp:
        reference = Path(tmp) / "ref.pt"
        torch.save(dict(state=model.state_dict(), grads=_grads(model), text=float(out["text_loss"]),
                        image=float(out["image_loss"])), reference)
        _spawn(_tp_worker, 2, Path(tmp) / "store", reference, Path(tmp) / "err")
        for r in range(2):
            errors = torch.load(Path(tmp) / f"err.{r}")
            assert len(errors) > 20
            bad = {k: v for k, v in errors.items() if v > 2e-5}   # fp32 inside a few reference ops
            assert not bad, sorted(bad.items())


_LOGGED = ("all_reduce", "reduce_scatter_tensor", "all_gather_into_tensor", "all_gather", "broadcast",
           "reduce_scatter", "barrier")


def _order_worker(rank, world, store, out):
    _init(rank, world, store)
    from cq_pretrain_b200.parallel import state as ps
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.train.trainer import Trainer
    ps.initialize(1, backend="gloo", device="cpu")
    cfg = _cfg()
    log = []
    originals = {name: getattr(dist, name) for name in _LOGGED}

    def wrap(name, fn):
        def logged(*args, **kwargs):
            t = args[0] if args and isinstance(args[0], torch.Tensor) else None
            log.append((name, tuple(t.shape) if t is not None else None, str(t.dtype) if t is not None else None))
            return fn(*args, **kwargs)
        return logged

    for name, fn in originals.items():
        setattr(dist, name, wrap(name, fn))
    try:
        trainer = Trainer(cfg, tp=1, lr=1e-3, ema_decay=0.9, device="cpu", dtype=torch.float32, seed=5,
                          bucket_size=30_000)
        images = 2 if rank == 0 else 0              # rank 1 has text only: no renderer branch
        host = synthetic_batch(cfg, 256, seed=21 + rank, pad_multiple=8, images=images)
        before = len(log)
        metrics = [trainer.train_step([host]) for _ in range(2)]
    finally:
        for name, fn in originals.items():
            setattr(dist, name, fn)
    torch.save(dict(log=log[before:], loss=[m["loss"] for m in metrics]), f"{out}.{rank}")
    dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_absent_renderer_branch_keeps_collective_order():
    with tempfile.TemporaryDirectory() as tmp:
        _spawn(_order_worker, 2, Path(tmp) / "store", Path(tmp) / "res")
        a, b = (torch.load(Path(tmp) / f"res.{r}") for r in range(2))
    assert a["log"] == b["log"] and len(a["log"]) > 4
    assert all(x == x for x in a["loss"] + b["loss"])


def _ema_worker(rank, world, store, root, out):
    _init(rank, world, store)
    from cq_pretrain_b200.parallel import state as ps
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.train import eval_snapshot
    from cq_pretrain_b200.train.trainer import Trainer, build_model
    st = ps.initialize(2, backend="gloo", device="cpu")
    cfg = _cfg()
    trainer = Trainer(cfg, tp=2, lr=1e-2, ema_decay=0.5, device="cpu", dtype=torch.float32, seed=5)
    host = synthetic_batch(cfg, 256, seed=31 + st.dp_rank, pad_multiple=16)
    for _ in range(3):
        trainer.train_step([host])
    online = {n: p.detach().clone() for n, p in trainer.model.named_parameters()}
    with trainer.ema.average_parameters():
        averaged = {n: p.detach().clone() for n, p in trainer.model.named_parameters()}
    restored = {n: p.detach().clone() for n, p in trainer.model.named_parameters()}
    eval_snapshot.save(Path(root) / "snap", trainer.model, 3, cfg, ema=trainer.ema)
    fresh = build_model(cfg, torch.device("cpu"), seed=99, dtype=torch.float32)
    eval_snapshot.load(Path(root) / "snap", fresh)
    loaded = dict(fresh.named_parameters())
    res = dict(
        restored=all(torch.equal(online[n], restored[n]) for n in online),
        renderer_moved=any(not torch.equal(online[n], averaged[n]) for n in online if n.startswith("renderer.")),
        backbone_online=all(torch.equal(online[n], averaged[n]) for n in online if not n.startswith("renderer.")),
        snapshot=all(torch.equal(loaded[n].detach(), averaged[n]) for n in averaged))
    torch.save(res, f"{out}.{rank}")
    dist.destroy_process_group()


@pytest.mark.timeout(900)
def test_ema_swap_and_eval_snapshot_round_trip_world4():
    with tempfile.TemporaryDirectory() as tmp:
        _spawn(_ema_worker, 4, Path(tmp) / "store", tmp, Path(tmp) / "res")
        for r in range(4):
            res = torch.load(Path(tmp) / f"res.{r}")
            assert all(res.values()), (r, res)
