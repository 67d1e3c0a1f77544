"""Inference-only weight snapshots (online backbone + EMA renderer), separate from restart state.

``save`` runs on every rank at an update boundary: the EMA weights are installed, DP rank 0 of
each TP rank writes ``model_tp_XXX.pt``, and rank 0 writes ``manifest.json`` (schema
``cq_eval_snapshot_v2``, kind ``inference_weights``) as the commit marker. Snapshots are
immutable: saving onto an existing commit with identical content is a no-op, different
content is an error. Rank-local failures are gathered collectively so no rank hangs
(reference ``utils/eval_snapshot.py:19-186``).
"""

from __future__ import annotations

import json
from contextlib import nullcontext
from pathlib import Path

import torch
import torch.distributed as dist

from ..parallel import state as ps
from .catalog import durable_json
from .checkpoint import _Files, topology

SCHEMA = "cq_eval_snapshot_v2"
KIND = "inference_weights"


def inspect_snapshot(path):
    root = Path(path)
    if root.is_symlink() or not root.is_dir():
        raise ValueError("evaluation snapshot must be a real directory")
    manifest = json.loads((root / "manifest.json").read_text())
    if manifest.get("schema") != SCHEMA or manifest.get("kind") != KIND:
        raise ValueError("unsupported evaluation snapshot manifest")
    step, tp = manifest["step"], manifest["topology"]["tp"]
    if type(step) is not int or step < 0 or type(tp) is not int or tp < 1:
        raise ValueError("invalid snapshot step or TP size")
    names = {f"model_tp_{i:03d}.pt" for i in range(tp)}
    files = manifest.get("files")
    if not isinstance(files, dict) or set(files) != names:
        raise ValueError("incomplete evaluation snapshot inventory")
    for name, size in files.items():
        shard = root / name
        if type(size) is not int or size <= 0 or shard.is_symlink() or not shard.is_file():
            raise ValueError(f"missing or invalid snapshot shard: {name}")
        if shard.stat().st_size != size:
            raise ValueError(f"truncated snapshot shard: {name}")
    return manifest


def _gather_errors(error, phase):
    if not dist.is_initialized():
        if error:
            raise RuntimeError(f"evaluation snapshot {phase} failed: {error}")
        return
    errors = [None] * dist.get_world_size()
    dist.all_gather_object(errors, error)
    failures = [f"rank {r}: {e}" for r, e in enumerate(errors) if e]
    if failures:
        raise RuntimeError(f"evaluation snapshot {phase} failed: " + "; ".join(failures))


def save(path, model, step, config, ema=None, provenance=None):
    root = Path(path)
    committed = (root / "manifest.json").exists()
    if dist.is_initialized():
        flags = [None] * dist.get_world_size()
        dist.all_gather_object(flags, committed)
        committed = any(flags)
    if committed:
        manifest = inspect_snapshot(root)
        if manifest["step"] != step or manifest["config"] != config.to_dict():
            raise FileExistsError(f"a different evaluation snapshot is committed at {root}")
        return manifest
    st = ps.state()
    error = None
    context = ema.average_parameters() if ema is not None else nullcontext()
    with context:
        try:
            root.mkdir(parents=True, exist_ok=True)
            if st.dp_rank == 0:
                files = _Files(root)
                files.write(files.model(st.tp_rank), model.state_dict())
        except Exception as exc:  # noqa: BLE001 - propagated collectively
            error = f"{type(exc).__name__}: {exc}"
        _gather_errors(error, "write")
    manifest = None
    if not dist.is_initialized() or dist.get_rank() == 0:
        files = {f"model_tp_{i:03d}.pt": (root / f"model_tp_{i:03d}.pt").stat().st_size for i in range(st.tp)}
        manifest = dict(schema=SCHEMA, kind=KIND, step=step, topology=topology(), config=config.to_dict(),
                        files=files, ema=(ema.metadata() if ema is not None else None), provenance=provenance or {})
        durable_json(root / "manifest.json", manifest)
    if dist.is_initialized():
        dist.barrier()
    return manifest


def load(path, model):
    """Load this TP rank's inference weights (same TP size as the snapshot)."""
    manifest = inspect_snapshot(path)
    if manifest["topology"]["tp"] != ps.tp_size():
        raise ValueError("snapshot TP differs; use checkpoint.initialize_model to reshard")
    state = torch.load(Path(path) / f"model_tp_{ps.tp_rank():03d}.pt", map_location="cpu", weights_only=False)
    with torch.no_grad():
        model.load_state_dict(state, strict=True)
    return manifest
