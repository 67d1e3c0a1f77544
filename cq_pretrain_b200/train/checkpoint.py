"""Atomic per-rank restart checkpoints with local FP32 Adam/master shards (schema 7 layout).

``save``: DP rank 0 of each TP rank writes ``model_tp_XXX.pt`` (bf16/fp32 model tensors), every
rank writes ``rank_XXXXX.pt`` (step, config, tp_rank, topology, CPU and device RNG states,
data cursor, optimizer shards, EMA shards), then rank 0 writes ``manifest.json`` (the commit
marker) after a barrier. ``load`` requires the identical TP/DP topology, config and training
state, restores model tensors (DP-broadcast from DP rank 0), optimizer shards, EMA and RNG.
``initialize_model`` is the model-only new stage and may change TP by exact resharding.
Reference: ``utils/checkpoint.py:15-204``. The device RNG is stored under ``device_rng``; the
reference's ``npu_rng`` key is accepted on load for files written by it.
"""

from __future__ import annotations

import json
import os
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


def _save_file(value, path):
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    with tmp.open("wb") as handle:
        torch.save(_cpu(value), handle)
        handle.flush()
        os.fsync(handle.fileno())
    os.replace(tmp, path)
    fsync_directory(path.parent)


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
    root = Path(path)
    if (root / "manifest.json").exists():
        raise FileExistsError(f"refusing to overwrite a committed checkpoint: {root}")
    root.mkdir(parents=True, exist_ok=True)
    st = ps.state()
    topo = topology()
    if st.dp_rank == 0:
        _save_file(model.state_dict(), root / f"model_tp_{st.tp_rank:03d}.pt")
    payload = dict(step=step, config=config.to_dict(), tp_rank=st.tp_rank, topology=topo,
                   cpu_rng=torch.get_rng_state(),
                   device_rng=torch.cuda.get_rng_state() if torch.cuda.is_available() and st.device.type == "cuda" else None,
                   schema=SCHEMA, data_state=data_state, optimizer=[optimizer.state_dict()])
    if ema is not None:
        payload["ema"] = ema.state_dict()
    _save_file(payload, root / f"rank_{_rank():05d}.pt")
    _barrier()
    if _rank() == 0:
        files = {name: (root / name).stat().st_size for name in shard_names(_world(), topo["tp"])}
        if any(size <= 0 for size in files.values()):
            raise RuntimeError("cannot commit an incomplete checkpoint")
        manifest = dict(schema=SCHEMA, step=step, world=_world(), topology=topo, config=config.to_dict(),
                        training_state=training_state, files=files)
        if ema is not None:
            manifest["ema"] = ema.metadata()
        durable_json(root / "manifest.json", manifest)
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
    root = Path(path)
    manifest = json.loads((root / "manifest.json").read_text())
    if manifest.get("schema") != SCHEMA:
        raise ValueError("unsupported checkpoint schema; refusing a partial optimizer restore")
    if ("ema" in manifest) != (ema is not None):
        raise ValueError("resume must preserve whether renderer EMA is enabled")
    if manifest["world"] != _world() or manifest["topology"] != topology():
        raise ValueError("resume requires the saved TP/DP topology")
    if manifest["config"] != config.to_dict():
        raise ValueError("resume model configuration differs from the checkpoint")
    if manifest.get("training_state") != training_state:
        raise ValueError("resume schedule, batch or data seed differs from the checkpoint")
    saved = torch.load(root / f"rank_{_rank():05d}.pt", map_location="cpu", weights_only=False)
    if saved.get("schema") != manifest["schema"]:
        raise ValueError("checkpoint shard and manifest schemas disagree")
    if ("ema" in saved) != ("ema" in manifest):
        raise ValueError("renderer EMA shard and manifest disagree")
    if data_state_out is not None:
        if saved.get("data_state") is None:
            raise ValueError("real-data resume needs a checkpoint with the consumed data state")
        data_state_out.update(saved["data_state"])
    st = ps.state()
    if st.dp_rank == 0:
        state = torch.load(root / f"model_tp_{saved['tp_rank']:03d}.pt", map_location="cpu", weights_only=False)
        with torch.no_grad():
            model.load_state_dict(state, strict=True)
    _broadcast_model(model)
    if len(saved["optimizer"]) != 1:
        raise ValueError("optimizer partition differs from the checkpoint")
    device_state = {k: v for k, v in saved["optimizer"][0].items()}
    optimizer.load_state_dict(_to_device(device_state, optimizer.shards[0]["master"].device))
    if ema is not None:
        ema.load_state_dict(_to_device(saved["ema"], optimizer.shards[0]["master"].device))
        if ema.metadata() != manifest["ema"]:
            raise ValueError("EMA metadata differs across checkpoint shards")
    torch.set_rng_state(saved["cpu_rng"])
    rng = saved.get("device_rng", saved.get("npu_rng"))
    if rng is not None and torch.cuda.is_available() and st.device.type == "cuda":
        torch.cuda.set_rng_state(rng)
    return saved["step"]


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

