"""Atomic per-rank restart checkpoints with local FP32 Adam/master shards (schema 7 layout).

``save``: DP rank 0 of each TP rank writes ``model_tp_XXX.pt`` (bf16/fp32 model tensors), every
rank writes ``rank_XXXXX.pt`` (step, config, tp_rank, topology, CPU and device RNG states,
data cursor, optimizer shards, EMA shards), then rank 0 writes ``manifest.json`` (the commit
marker) after a barrier. ``load`` requires the identical TP/DP topology, config and training
state, restores model tensors (DP-broadcast from DP rank 0), optimizer shards, EMA and RNG.
``initialize_model`` is the model-only new stage and may change TP by exact resharding. A resume
compares a ``RunIdentity`` (world, topology, config, training state, EMA presence) of the
manifest with the running job and reports every difference in one error.
Reference: ``utils/checkpoint.py:15-204``. The device RNG is stored under ``device_rng``; the
reference's ``npu_rng`` key is accepted on load for files written by it.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, fields
from pathlib import Path

import torch
import torch.distributed as dist

from ..parallel import state as ps
from .catalog import SCHEMA, durable_json, fsync_directory, shard_names


def _cpu(value):
    if isinstance(value, torch.Tensor):
        return value.detach().cpu().clone()
    if isinstance(value, dict):
        return {k: _cpu(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return type(value)(_cpu(v) for v in value)
    return value


def topology():
    st = ps.state()
    return dict(world=st.world, tp=st.tp, dp=st.dp, pp=1, cp=1)


def _barrier():
    if dist.is_initialized():
        dist.barrier()


def _rank():
    return dist.get_rank() if dist.is_initialized() else 0


def _world():
    return dist.get_world_size() if dist.is_initialized() else 1


class _Files:
    """Names and crash-safe writers of one checkpoint directory (schema 7 file layout)."""

    def __init__(self, root):
        self.root = Path(root)
        self.manifest = self.root / "manifest.json"

    def model(self, tp_rank):
        return self.root / f"model_tp_{tp_rank:03d}.pt"

    def rank(self, rank):
        return self.root / f"rank_{rank:05d}.pt"

    def begin(self):
        if self.manifest.exists():
            raise FileExistsError(f"{self.root} is already committed; a checkpoint is never overwritten")
        self.root.mkdir(parents=True, exist_ok=True)

    def write(self, path, value):
        scratch = path.with_name(path.name + ".partial")
        with scratch.open("wb") as handle:
            torch.save(_cpu(value), handle)
            handle.flush()
            os.fsync(handle.fileno())
        os.replace(scratch, path)
        fsync_directory(self.root)

    def commit(self, manifest):
        durable_json(self.manifest, manifest)

    def read_manifest(self):
        return json.loads(self.manifest.read_text())

    def load(self, path):
        return torch.load(path, map_location="cpu", weights_only=False)


@dataclass
class RunIdentity:
    """What a restart must reproduce exactly: rank layout, model config, training schedule and
    data identity, and whether a renderer EMA is kept."""

    world: int
    topology: dict
    config: dict
    training_state: object
    ema: bool

    @classmethod
    def current(cls, config, training_state, ema):
        return cls(_world(), topology(), config.to_dict(), training_state, ema is not None)

    @classmethod
    def saved(cls, manifest):
        return cls(manifest.get("world"), manifest.get("topology"), manifest.get("config"),
                   manifest.get("training_state"), "ema" in manifest)

    def mismatches(self, now):
        out = []
        for f in fields(self):
            then, current = getattr(self, f.name), getattr(now, f.name)
            if then == current:
                continue
            if isinstance(then, dict) and isinstance(current, dict):
                keys = sorted(k for k in then.keys() | current.keys() if then.get(k) != current.get(k))
                out.append(f"{f.name} differs in {keys[:8]}")
            else:
                out.append(f"{f.name} was {then!r}, now {current!r}")
        return out


def validation_probes(model, optimizer):
    """16 strided samples of every parameter, master and Adam-state tensor (restart bit-equality checks)."""
    values, layout = [], []

    def add(name, tensor):
        if not tensor.numel():
            return
        flat = tensor.detach().flatten()
        picked = flat[:: max(1, flat.numel() // 16)][:16].float()
        values.append(picked)
        layout.append((name, tuple(tensor.shape), picked.numel()))

    for name, p in model.named_parameters():
        add("model/" + name, p)
    for i, shard in enumerate(optimizer.shards):
        for key in ("master", "exp_avg", "exp_avg_sq"):
            add(f"{key}/{i}", shard[key])
    return dict(layout=layout, values=torch.cat(values).cpu())


def save(path, model, optimizer, step, config, training_state=None, data_state=None, ema=None):
    """Write this rank's shards; rank 0 commits the manifest once every rank has written."""
    files = _Files(path)
    files.begin()
    st = ps.state()
    if hasattr(optimizer, "wait_params"):
        optimizer.wait_params()             # parameters of the last update must have arrived
    identity = RunIdentity.current(config, training_state, ema)
    if st.dp_rank == 0:                      # one model shard per TP rank
        files.write(files.model(st.tp_rank), model.state_dict())
    cuda = torch.cuda.is_available() and st.device.type == "cuda"
    shard = dict(step=step, config=identity.config, tp_rank=st.tp_rank, topology=identity.topology,
                 schema=SCHEMA, cpu_rng=torch.get_rng_state(), device_rng=torch.cuda.get_rng_state() if cuda else None,
                 data_state=data_state, optimizer=[optimizer.state_dict()])
    if ema is not None:
        shard["ema"] = ema.state_dict()
    files.write(files.rank(_rank()), shard)
    _barrier()
    if _rank() == 0:
        sizes = {}
        for name in shard_names(identity.world, identity.topology["tp"]):
            size = (files.root / name).stat().st_size
            if size <= 0:
                raise RuntimeError(f"{name} is empty; the checkpoint is not committed")
            sizes[name] = size
        manifest = dict(schema=SCHEMA, step=step, world=identity.world, topology=identity.topology,
                        config=identity.config, training_state=training_state, files=sizes)
        if ema is not None:
            manifest["ema"] = ema.metadata()
        files.commit(manifest)
    _barrier()


def _broadcast_model(model):
    st = ps.state()
    if st.dp <= 1:
        return
    src = st.dp_ranks[0]
    for tensor in model.state_dict().values():
        if isinstance(tensor, torch.Tensor):
            dist.broadcast(tensor, src=src, group=st.dp_group)


def load(path, model, optimizer, config, training_state=None, data_state_out=None, ema=None):
    """Restore a restart checkpoint; every incompatibility is collected and reported at once."""
    files = _Files(path)
    manifest = files.read_manifest()
    shard = files.load(files.rank(_rank()))
    problems = []
    if manifest.get("schema") != SCHEMA:
        problems.append(f"schema {manifest.get('schema')!r} (this build reads {SCHEMA})")
    if shard.get("schema") != manifest.get("schema"):
        problems.append("the rank shard and the manifest carry different schemas")
    problems += RunIdentity.saved(manifest).mismatches(RunIdentity.current(config, training_state, ema))
    if ("ema" in shard) != ("ema" in manifest):
        problems.append("the rank shard and the manifest disagree on the renderer EMA")
    if data_state_out is not None and shard.get("data_state") is None:
        problems.append("no consumed-data cursor was saved, so a corpus run cannot resume from it")
    if len(shard.get("optimizer", ())) != 1:
        problems.append("the optimizer partition differs")
    if problems:
        raise ValueError(f"cannot resume from {files.root}: " + "; ".join(problems))
    if data_state_out is not None:
        data_state_out.update(shard["data_state"])
    st = ps.state()
    if st.dp_rank == 0:
        with torch.no_grad():
            model.load_state_dict(files.load(files.model(shard["tp_rank"])), strict=True)
    _broadcast_model(model)
    device = optimizer.shards[0]["master"].device
    optimizer.load_state_dict(_to_device(dict(shard["optimizer"][0]), device))
    if ema is not None:
        ema.load_state_dict(_to_device(shard["ema"], device))
        if ema.metadata() != manifest["ema"]:
            raise ValueError("the restored EMA's metadata differs from the manifest's")
    torch.set_rng_state(shard["cpu_rng"])
    rng = shard.get("device_rng", shard.get("npu_rng"))
    if rng is not None and torch.cuda.is_available() and st.device.type == "cuda":
        torch.cuda.set_rng_state(rng)
    return shard["step"]


def _to_device(value, device):
    if isinstance(value, torch.Tensor):
        return value.to(device)
    if isinstance(value, dict):
        return {k: _to_device(v, device) for k, v in value.items()}
    if isinstance(value, list):
        return [_to_device(v, device) for v in value]
    return value


EXECUTION_FIELDS = {
    "checkpoint_backbone", "checkpoint_dit", "checkpoint_backbone_layers", "checkpoint_dit_layers", "ce_chunk",
    "keep_attention_activations", "preserve_documents", "long_document_policy", "generation_token_budget",
    "generation_microbatch_images", "i2t_image_loss_probability", "visual_uncond_probability", "cfg_null_condition",
    "image_condition_queries", "visual_query_mode", "visual_cache", "gdn_backend"}


def initialization_model_config(config: dict) -> dict:
    """Config fields that define learned tensors; execution/packing settings may change in a new stage."""
    return {k: v for k, v in config.items() if k not in EXECUTION_FIELDS}


def initialize_model(path, model, config):
    """Model-only new stage (fresh optimizer and data cursor); TP may differ (exact reshard)."""
    root = Path(path)
    manifest = json.loads((root / "manifest.json").read_text())
    from .eval_snapshot import SCHEMA as SNAPSHOT_SCHEMA
    if manifest.get("schema") not in (SCHEMA, SNAPSHOT_SCHEMA):
        raise ValueError("unsupported model initialization schema")
    if manifest["config"].keys() != config.to_dict().keys():
        raise ValueError("initialization configuration fields differ from the checkpoint")
    saved, current = initialization_model_config(manifest["config"]), initialization_model_config(config.to_dict())
    if saved != current:
        changed = sorted(k for k in saved.keys() | current.keys() if saved.get(k) != current.get(k))
        raise ValueError(f"initialization semantic model config differs: {changed}")
    source_tp = manifest["topology"]["tp"]
    st = ps.state()
    if st.dp_rank == 0:
        def read(i):
            name = f"model_tp_{i:03d}.pt"
            if (root / name).stat().st_size != manifest["files"][name]:
                raise ValueError("initialization shard size mismatch")
            return torch.load(root / name, map_location="cpu", weights_only=False, mmap=True)

        if source_tp == st.tp:
            state = read(st.tp_rank)
        else:
            from .reshard import reshard_state
            state = reshard_state([read(i) for i in range(source_tp)], model, st.tp, st.tp_rank)
        with torch.no_grad():
            model.load_state_dict(state, strict=True)
    _broadcast_model(model)
    return dict(path=str(root), source_step=manifest["step"], source_tp=source_tp, target_tp=st.tp,
                restored=["model"], new_stage=True, optimizer="fresh", data_cursor="new dataset start")

