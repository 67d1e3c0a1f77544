"""Small file-system primitives shared by the launcher, supervisor, tuner and checkpoints.

* ``atomic_json(path, value, durable=False)``: the JSON text goes to a uniquely named sibling
  created with ``mkstemp`` and is moved over ``path`` with ``os.replace``, so readers see the old
  or the new document, never a torn one. ``durable=True`` also fsyncs the file before the move
  and the directory after it (crash-safe commit markers).
* ``read_json(path)``: the document, or ``None`` while it does not exist yet.
* ``wait_files(paths, timeout)``: polls with a growing interval (50 ms up to 1 s) until every
  path exists, and names the missing ones when the deadline passes.
"""

from __future__ import annotations

import json
import os
import tempfile
import time
from pathlib import Path


def fsync_directory(path):
    """Flush a directory entry table (after a rename or unlink inside it)."""
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def atomic_json(path, value, durable=False):
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    text = json.dumps(value, indent=2) + "\n"
    fd, scratch = tempfile.mkstemp(prefix=f".{target.name}.", dir=target.parent)
    try:
        with os.fdopen(fd, "w") as handle:
            handle.write(text)
            if durable:
                handle.flush()
                os.fsync(handle.fileno())
        os.replace(scratch, target)
    except BaseException:
        if os.path.exists(scratch):
            os.unlink(scratch)
        raise
    if durable:
        fsync_directory(target.parent)
    return target


def read_json(path):
    try:
        with open(path) as handle:
            return json.load(handle)
    except FileNotFoundError:
        return None


def wait_files(paths, timeout=1200.0, first_poll=0.05, max_poll=1.0):
    pending = [Path(p) for p in paths]
    give_up = time.monotonic() + timeout
    poll = first_poll
    while True:
        pending = [p for p in pending if not p.is_file()]
        if not pending:
            return
        if time.monotonic() >= give_up:
            raise TimeoutError(f"still missing after {timeout:.0f} s: {', '.join(str(p) for p in pending)}")
        time.sleep(poll)
        poll = min(max_poll, poll * 2)
