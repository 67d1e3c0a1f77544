"""Committed-checkpoint discovery and bounded retention (no accelerator imports).

A checkpoint is ``<root>/step_XXXXXXX/`` holding ``model_tp_{i:03d}.pt`` (one per TP rank),
``rank_{r:05d}.pt`` (one per rank) and ``manifest.json``, written last as the commit marker
with the exact byte size of every shard. Directory layout, file names and schema number
follow the reference format (``utils/checkpoint_catalog.py:8-110``) so tooling interoperates.
"""

from __future__ import annotations

import json
import os
import re
import shutil
from pathlib import Path

SCHEMA = 7


def fsync_directory(path):
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def durable_json(path, value):
    """Write JSON atomically: temp file, fsync, rename, fsync the directory."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    with tmp.open("w") as handle:
        json.dump(value, handle, indent=2)
        handle.write("\n")
        handle.flush()
        os.fsync(handle.fileno())
    os.replace(tmp, path)
    fsync_directory(path.parent)


def shard_names(world, tp):
    if not isinstance(world, int) or not isinstance(tp, int) or tp < 1 or world < tp or world % tp:
        raise ValueError("invalid checkpoint topology")
    return [f"model_tp_{i:03d}.pt" for i in range(tp)] + [f"rank_{i:05d}.pt" for i in range(world)]


def inspect_checkpoint(path):
    """Validate a committed checkpoint without loading tensors; returns its manifest."""
    path = Path(path)
    if path.is_symlink() or not path.is_dir():
        raise ValueError("checkpoint must be a real directory")
    manifest = json.loads((path / "manifest.json").read_text())
    if manifest.get("schema") != SCHEMA:
        raise ValueError("unsupported checkpoint schema")
    step = manifest["step"]
    if not isinstance(step, int) or step < 0 or path.name != f"step_{step:07d}":
        raise ValueError("checkpoint step/directory mismatch")
    topo = manifest["topology"]
    names = shard_names(manifest["world"], topo["tp"])
    if topo["dp"] * topo["tp"] != manifest["world"]:
        raise ValueError("invalid saved DP topology")
    sizes = manifest.get("files")
    if not isinstance(sizes, dict) or set(sizes) != set(names):
        raise ValueError("incomplete checkpoint inventory")
    for name in names:
        shard = path / name
        if shard.is_symlink() or not shard.is_file() or shard.stat().st_size == 0:
            raise ValueError(f"missing/empty shard: {name}")
        if shard.stat().st_size != sizes[name]:
            raise ValueError(f"truncated shard: {name}")
    return manifest


def checkpoint_directories(root):
    root = Path(root)
    return sorted((p for p in root.glob("step_*") if re.fullmatch(r"step_\d{7,}", p.name) and p.is_dir()
                   and not p.is_symlink()), key=lambda p: int(p.name[5:]), reverse=True)


def discover(root):
    committed, rejected = [], []
    for path in checkpoint_directories(root):
        try:
            manifest = inspect_checkpoint(path)
        except (OSError, ValueError, KeyError, TypeError) as error:
            rejected.append(dict(path=str(path), reason=str(error), committed=(path / "manifest.json").exists()))
        else:
            committed.append((path, manifest))
    return committed, rejected


def latest(root):
    """Newest intact committed checkpoint; refuses a silent restart if only corrupt commits exist."""
    committed, rejected = discover(root)
    if not committed and any(item["committed"] for item in rejected):
        raise RuntimeError(f"no intact committed checkpoint; refusing to restart from scratch: {rejected}")
    return (str(committed[0][0]) if committed else None), rejected


def prune(root, keep):
    """Keep the ``keep`` newest intact checkpoints (call with exclusive ownership, after a commit)."""
    if keep < 1:
        raise ValueError("retain at least one checkpoint")
    committed, _ = discover(root)
    if not committed:
        raise RuntimeError("refusing cleanup without an intact committed checkpoint")
    retained = {p for p, _ in committed[:keep]}
    removed = []
    for path in checkpoint_directories(root):
        if path not in retained:
            shutil.rmtree(path)
            removed.append(str(path))
    fsync_directory(root)
    return removed


def remove_incomplete(root):
    """Remove uncommitted attempts (no manifest); only while no writer is running."""
    removed = []
    for path in checkpoint_directories(root):
        if not (path / "manifest.json").exists():
            shutil.rmtree(path)
            removed.append(str(path))
    return removed
