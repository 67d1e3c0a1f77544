"""Checkpoint/resume, corruption handling, TP resharding and eval snapshots (CPU, gloo ranks)."""

import json
import os
import tempfile
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.train import catalog


def _cfg():
    return tiny_config(layers=4, dit_layers=1, vocab_size=256, width=128, ffn=256, heads=4, kv_heads=2, head_dim=32,
                       mrope_section=(2, 1, 1), linear_heads=2, linear_head_dim=32, dit_width=64, dit_heads=2,
                       dit_ffn=128)


def _init(rank, world, tp, store):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    from cq_pretrain_b200.parallel import state as ps
    return ps.initialize(tp, backend="gloo", device="cpu")


def _trainer(tp):
    from cq_pretrain_b200.train.trainer import Trainer
    return Trainer(_cfg(), tp=tp, lr=1e-3, ema_decay=0.9, device="cpu", dtype=torch.float32, seed=5)


def _batch(st, length=256):
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    return synthetic_batch(_cfg(), length, seed=11 + st.dp_rank, pad_multiple=8 * st.tp)


def _restart_worker(rank, world, tp, store, root, out):
    st = _init(rank, world, tp, store)
    from cq_pretrain_b200.train import checkpoint as C
    torch.manual_seed(0)
    trainer = _trainer(tp)
    batch = _batch(st)
    # three uninterrupted steps
    for _ in range(3):
        trainer.train_step([batch])
    probe_a = C.validation_probes(trainer.model, trainer.optimizer)["values"]
    # fresh run: two steps, checkpoint, fresh process state, resume, one step
    trainer2 = _trainer(tp)
    for _ in range(2):
        trainer2.train_step([batch])
    C.save(Path(root) / "step_0000002", trainer2.model, trainer2.optimizer, 2, trainer2.cfg,
           training_state={"seed": 1}, data_state={"cursor": 7}, ema=trainer2.ema)
    trainer3 = _trainer(tp)
    data = {}
    step = C.load(Path(root) / "step_0000002", trainer3.model, trainer3.optimizer, trainer3.cfg,
                  training_state={"seed": 1}, data_state_out=data, ema=trainer3.ema)
    trainer3.step_index = step
    trainer3.train_step([batch])
    probe_b = C.validation_probes(trainer3.model, trainer3.optimizer)["values"]
    if rank == 0:
        torch.save(dict(a=probe_a, b=probe_b, step=step, data=data), out)
    dist.destroy_process_group()


def _spawn(fn, world, *args):
    mp.start_processes(fn, args=(world, *args), nprocs=world, start_method="spawn", join=True)


@pytest.mark.timeout(600)
def test_restart_is_bitwise_identical_tp2():
    with tempfile.TemporaryDirectory() as tmp:
        store, root, out = Path(tmp) / "store", Path(tmp) / "ckpt", Path(tmp) / "out.pt"
        _spawn(_restart_worker, 2, 2, str(store), str(root), str(out))
        result = torch.load(out)
        assert result["step"] == 2 and result["data"] == {"cursor": 7}
        torch.testing.assert_close(result["a"], result["b"], atol=0, rtol=0)
        manifest = catalog.inspect_checkpoint(root / "step_0000002")
        assert manifest["topology"]["tp"] == 2 and manifest["world"] == 2


def _reshard_worker(rank, world, tp, store, root, out):
    st = _init(rank, world, tp, store)
    from cq_pretrain_b200.train import checkpoint as C
    trainer = _trainer(tp)
    batch = _batch(st)
    trainer.train_step([batch])
    C.save(Path(root) / "step_0000001", trainer.model, trainer.optimizer, 1, trainer.cfg, ema=trainer.ema)
    # full (TP-gathered) reference of every tensor, assembled on rank 0 via all_gather of shards
    shards = {}
    for name, p in trainer.model.state_dict(keep_vars=True).items():
        parts = [torch.empty_like(p.detach()) for _ in range(world)]
        dist.all_gather(parts, p.detach().contiguous())
        shards[name] = parts
    if rank == 0:
        torch.save({k: [t.clone() for t in v] for k, v in shards.items()}, out)
    dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_tp2_checkpoint_initializes_tp1_model_exactly():
    with tempfile.TemporaryDirectory() as tmp:
        store, root, out = Path(tmp) / "store", Path(tmp) / "ckpt", Path(tmp) / "parts.pt"
        _spawn(_reshard_worker, 2, 2, str(store), str(root), str(out))
        from cq_pretrain_b200.parallel import state as ps
        from cq_pretrain_b200.train import checkpoint as C
        from cq_pretrain_b200.train.trainer import build_model
        ps.set_state_for_tests(ps.ParallelState())
        model = build_model(_cfg(), torch.device("cpu"), 9, torch.float32)
        info = C.initialize_model(root / "step_0000001", model, _cfg())
        assert info["source_tp"] == 2 and info["target_tp"] == 1
        parts = torch.load(out)
        from cq_pretrain_b200.train.reshard import reshard_tensor
        state = model.state_dict(keep_vars=True)
        for name, value in state.items():
            expect = reshard_tensor(parts[name], value, 1, 0)
            torch.testing.assert_close(value.detach(), expect, atol=0, rtol=0, msg=name)


def test_catalog_rejects_corrupt_and_prunes(tmp_path):
    def fake(step, truncate=False, commit=True):
        d = tmp_path / f"step_{step:07d}"
        d.mkdir()
        files = {}
        for name in catalog.shard_names(1, 1):
            (d / name).write_bytes(b"x" * 10)
            files[name] = 10
        if truncate:
            (d / "rank_00000.pt").write_bytes(b"x")
        if commit:
            catalog.durable_json(d / "manifest.json", dict(schema=catalog.SCHEMA, step=step, world=1,
                                                           topology=dict(tp=1, dp=1), files=files))
        return d

    fake(1)
    fake(2, truncate=True)
    fake(3, commit=False)
    path, rejected = catalog.latest(tmp_path)
    assert path.endswith("step_0000001")
    assert {Path(r["path"]).name for r in rejected} == {"step_0000002", "step_0000003"}
    assert catalog.remove_incomplete(tmp_path)[0].endswith("step_0000003")
    fake(4)
    removed = catalog.prune(tmp_path, 1)
    assert sorted(Path(p).name for p in removed) == ["step_0000001", "step_0000002"]


def test_latest_refuses_only_corrupt_commits(tmp_path):
    d = tmp_path / "step_0000005"
    d.mkdir()
    (d / "manifest.json").write_text(json.dumps(dict(schema=catalog.SCHEMA, step=5, world=1,
                                                     topology=dict(tp=1, dp=1), files={})))
    with pytest.raises(RuntimeError):
        catalog.latest(tmp_path)


def test_validation_probes_layout():
    import torch
    from cq_pretrain_b200.config import tiny_config
    from cq_pretrain_b200.train.checkpoint import validation_probes
    from cq_pretrain_b200.train.trainer import Trainer
    trainer = Trainer(tiny_config(), tp=1, lr=1e-3, device="cpu", dtype=torch.float32)
    probes = validation_probes(trainer.model, trainer.optimizer)
    names = [name for name, _, _ in probes["layout"]]
    assert names[0].startswith("model/") and any(n.startswith("exp_avg/") for n in names)
    assert probes["values"].numel() == sum(c for _, _, c in probes["layout"])
    again = validation_probes(trainer.model, trainer.optimizer)
    assert torch.equal(probes["values"], again["values"])


def _dp_worker(rank, world, tp, store, out):
    st = _init(rank, world, tp, store)
    from cq_pretrain_b200.train.trainer import Trainer
    batch = _batch(st)
    results = {}
    for overlap in (False, True):
        trainer = Trainer(_cfg(), tp=tp, lr=1e-3, ema_decay=0.9, device="cpu", dtype=torch.float32, seed=5,
                          overlap=overlap)
        losses = [trainer.train_step([batch])["loss"] for _ in range(3)]
        params = torch.cat([p.detach().flatten() for p in trainer.model.parameters()])
        results[overlap] = (losses, params)
    gathered = [None] * world
    dist.all_gather_object(gathered, results[True][1])
    if rank == 0:
        torch.save(dict(plain=results[False], overlap=results[True], ranks=gathered), out)
    dist.destroy_process_group()


def test_data_parallel_overlap_matches_serial_dp2():
    with tempfile.TemporaryDirectory() as tmp:
        out = Path(tmp) / "dp.pt"
        _spawn(_dp_worker, 2, 1, str(Path(tmp) / "store"), str(out))
        r = torch.load(out, weights_only=False)
    assert r["plain"][0] == r["overlap"][0]
    assert torch.equal(r["plain"][1], r["overlap"][1])
    assert torch.equal(r["ranks"][0], r["ranks"][1])   # DP replicas hold identical parameters
