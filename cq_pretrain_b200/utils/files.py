"""Atomic JSON writes and file synchronisation helpers (reference ``utils/file_sync.py``)."""

from __future__ import annotations

import json
import os
import time
from pathlib import Path


def atomic_json(path, value):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(f".tmp-{os.getpid()}")
    tmp.write_text(json.dumps(value, indent=2) + "\n")
    tmp.replace(path)


def read_json(path):
    try:
        return json.loads(Path(path).read_text())
    except FileNotFoundError:
        return None


def wait_files(paths, timeout=1200, interval=0.2):
    deadline = time.monotonic() + timeout
    paths = [Path(p) for p in paths]
    while not all(p.is_file() for p in paths):
        if time.monotonic() > deadline:
            raise TimeoutError(f"missing files: {[str(p) for p in paths if not p.exists()]}")
        time.sleep(interval)
