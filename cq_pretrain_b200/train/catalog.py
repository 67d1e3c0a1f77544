"""The checkpoint directory as a catalogue: scan, verify, pick the newest, retain, sweep.

On-disk format (kept so that shards written by either framework are interchangeable): one
directory ``step_XXXXXXX`` per save holding ``model_tp_{i:03d}.pt`` per TP rank,
``rank_{r:05d}.pt`` per rank and ``manifest.json`` (schema 7) with ``step``, ``world``,
``topology`` {tp, dp, ...} and ``files`` {name: byte size}. The manifest is written last and is
the commit marker.

``CheckpointStore(root).scan()`` classifies every step directory as *committed* (manifest and
every listed shard present at its recorded size), *corrupt* (a manifest exists but something is
wrong) or *partial* (no manifest: an interrupted save). The policies act on that classification:

* ``newest()``: the newest committed checkpoint; raises instead of returning ``None`` when
  commits exist but none is intact, so a run never silently restarts from scratch;
* ``retain(keep)``: deletes everything except the ``keep`` newest committed checkpoints;
* ``sweep_partial()``: deletes interrupted saves (only while no writer runs).

The module-level ``latest`` / ``prune`` / ``remove_incomplete`` / ``inspect_checkpoint`` are the
public entry points (reference ``utils/checkpoint_catalog.py:82-110`` names).
"""

from __future__ import annotations

import json
import re
import shutil
from dataclasses import dataclass, field
from pathlib import Path

from ..utils.files import atomic_json, fsync_directory

SCHEMA = 7
_STEP_DIR = re.compile(r"step_(\d{7,})")


def shard_names(world, tp):
    """File inventory of a checkpoint saved by ``world`` ranks at tensor parallelism ``tp``."""
    if not (isinstance(world, int) and isinstance(tp, int)) or tp < 1 or world < tp or world % tp:
        raise ValueError(f"no TP x DP layout has world {world} and TP {tp}")
    return [f"model_tp_{i:03d}.pt" for i in range(tp)] + [f"rank_{r:05d}.pt" for r in range(world)]


def durable_json(path, value):
    """Crash-safe JSON commit: fsynced file, atomic rename, fsynced directory."""
    return atomic_json(path, value, durable=True)


def _problems(path: Path, manifest: dict) -> list:
    """Everything that keeps ``path`` from being a usable committed checkpoint."""
    if manifest.get("schema") != SCHEMA:
        return [f"schema {manifest.get('schema')!r}, expected {SCHEMA}"]
    step, world, topo, sizes = (manifest.get(k) for k in ("step", "world", "topology", "files"))
    found = []
    if not isinstance(step, int) or path.name != f"step_{step:07d}":
        found.append(f"directory name does not match step {step!r}")
    if not isinstance(topo, dict) or topo.get("tp", 0) * topo.get("dp", 0) != world:
        return found + [f"topology {topo!r} does not multiply to world {world!r}"]
    try:
        expected = shard_names(world, topo["tp"])
    except ValueError as error:
        return found + [str(error)]
    if not isinstance(sizes, dict) or sorted(sizes) != sorted(expected):
        return found + ["the manifest's file inventory does not match the topology"]
    for name in expected:
        shard = path / name
        if shard.is_symlink() or not shard.is_file():
            found.append(f"{name} is missing")
        elif shard.stat().st_size in (0, None) or shard.stat().st_size != sizes[name]:
            found.append(f"{name} has {shard.stat().st_size} bytes, the manifest says {sizes[name]}")
    return found


@dataclass
class Entry:
    path: Path
    step: int
    state: str                     # "committed", "corrupt" or "partial"
    manifest: dict | None = None
    problems: list = field(default_factory=list)


class CheckpointStore:
    def __init__(self, root):
        self.root = Path(root)

    def scan(self):
        """Every ``step_*`` directory, newest first, with its classification."""
        entries = []
        if not self.root.is_dir():
            return entries
        for child in self.root.iterdir():
            match = _STEP_DIR.fullmatch(child.name)
            if not match or child.is_symlink() or not child.is_dir():
                continue
            entry = Entry(child, int(match.group(1)), "partial")
            marker = child / "manifest.json"
            if marker.exists():
                try:
                    entry.manifest = json.loads(marker.read_text())
                    entry.problems = _problems(child, entry.manifest)
                except (OSError, ValueError, TypeError, AttributeError) as error:
                    entry.problems = [f"unreadable manifest: {error}"]
                entry.state = "corrupt" if entry.problems else "committed"
            entries.append(entry)
        entries.sort(key=lambda e: e.step, reverse=True)
        return entries

    def committed(self):
        return [e for e in self.scan() if e.state == "committed"]

    def newest(self):
        """``(path or None, [rejected entries as dicts])``."""
        entries = self.scan()
        good = [e for e in entries if e.state == "committed"]
        rejected = [dict(path=str(e.path), reason="; ".join(e.problems) or "no manifest (interrupted save)",
                         committed=e.state == "corrupt") for e in entries if e.state != "committed"]
        if not good and any(e.state == "corrupt" for e in entries):
            raise RuntimeError(f"committed checkpoints exist under {self.root} but none is intact; "
                               f"refusing to start over: {rejected}")
        return (str(good[0].path) if good else None), rejected

    def retain(self, keep):
        if keep < 1:
            raise ValueError("retention must keep at least one checkpoint")
        entries = self.scan()
        keep_paths = {e.path for e in [e for e in entries if e.state == "committed"][:keep]}
        if not keep_paths:
            raise RuntimeError("no intact committed checkpoint: nothing is deleted")
        gone = []
        for e in entries:
            if e.path not in keep_paths:
                shutil.rmtree(e.path)
                gone.append(str(e.path))
        fsync_directory(self.root)
        return gone

    def sweep_partial(self):
        gone = []
        for e in self.scan():
            if e.state == "partial":
                shutil.rmtree(e.path)
                gone.append(str(e.path))
        return gone


def inspect_checkpoint(path):
    """The manifest of an intact committed checkpoint (``ValueError`` listing what is wrong otherwise)."""
    path = Path(path)
    if path.is_symlink() or not path.is_dir():
        raise ValueError(f"{path} is not a checkpoint directory")
    manifest = json.loads((path / "manifest.json").read_text())
    problems = _problems(path, manifest)
    if problems:
        raise ValueError(f"{path}: " + "; ".join(problems))
    return manifest


def latest(root):
    return CheckpointStore(root).newest()


def prune(root, keep):
    return CheckpointStore(root).retain(keep)


def remove_incomplete(root):
    return CheckpointStore(root).sweep_partial()
