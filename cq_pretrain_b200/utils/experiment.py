"""Source identity: sha256 of every framework source file (node agreement, run records)."""

from __future__ import annotations

import hashlib
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SUFFIXES = (".py", ".cu", ".cuh", ".cpp", ".h", ".yaml", ".json", ".sh")


def source_hashes(root=ROOT):
    root = Path(root)
    paths = sorted(p for p in root.rglob("*") if p.is_file() and p.suffix in SUFFIXES and "_build" not in p.parts
                   and "__pycache__" not in p.parts)
    return {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in paths}


def source_digest(root=ROOT):
    h = hashlib.sha256()
    for name, digest in source_hashes(root).items():
        h.update(f"{name}:{digest}\n".encode())
    return h.hexdigest()
