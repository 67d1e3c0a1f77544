"""Corpus catalogs and the DP-sharded, exactly-resumable document stream.

* ``Catalog``: documents from JSONL files or Parquet tables (one document per row, the
  ``elements`` column holding the element list as JSON), validated against a manifest
  (``COMPLETE`` marker, row counts, sha256 per file) when one is present.
* ``permute``: a constant-memory Feistel bijection over block indices, keyed by (seed, epoch),
  so shuffling needs no index table (reference ``data/catalog.py:19-155``).
* ``DocumentStream``: walks shuffled blocks of ``block_rows`` rows, assigning blocks to DP ranks
  round-robin; its cursor ``{epoch, block, row}`` plus a signature (snapshot, seed, rank) is the
  resumable state, and a resumed stream must present the same signature
  (reference ``data/stream.py:19-256``).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np


def _round(x, key, bits):
    h = hashlib.sha256(f"{key}:{x}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << bits) - 1)


def permute(index, n, seed, epoch, rounds=4):
    """Bijective shuffle of ``range(n)``: balanced Feistel network on the next even bit width with cycle walking."""
    if not 0 <= index < n:
        raise IndexError(index)
    bits = max(2, (n - 1).bit_length())
    bits += bits % 2
    half = bits // 2
    mask = (1 << half) - 1
    x = index
    while True:
        left, right = x >> half, x & mask
        for r in range(rounds):
            left, right = right, left ^ _round(right, f"{seed}:{epoch}:{r}", half)
        x = (left << half) | right
        if x < n:
            return x


class Catalog:
    def __init__(self, root):
        self.root = Path(root)
        manifest = self.root / "manifest.json"
        self.manifest = json.loads(manifest.read_text()) if manifest.exists() else None
        if self.manifest is not None:
            if not (self.root / "COMPLETE").exists():
                raise ValueError("corpus snapshot is not COMPLETE")
            for entry in self.manifest["files"]:
                path = self.root / entry["path"]
                if hashlib.sha256(path.read_bytes()).hexdigest() != entry["sha256"]:
                    raise ValueError(f"corpus file changed: {entry['path']}")
            files = [self.root / e["path"] for e in self.manifest["files"]]
        else:
            files = sorted(list(self.root.glob("*.jsonl")) + list(self.root.glob("*.parquet")))
        self.rows = []
        for f in files:
            if f.suffix == ".jsonl":
                self.rows.extend(json.loads(line) for line in f.read_text().splitlines() if line.strip())
            else:
                import pyarrow.parquet as pq
                table = pq.read_table(f).to_pylist()
                for row in table:
                    if isinstance(row.get("elements"), str):
                        row["elements"] = json.loads(row["elements"])
                    self.rows.append(row)
        for row in self.rows:
            for e in row["elements"]:
                if e["type"] == "text":
                    e["input_ids"] = np.asarray(e["input_ids"], dtype=np.int64)
        self.snapshot = self.manifest.get("snapshot", "unversioned") if self.manifest else "unversioned"

    def __len__(self):
        return len(self.rows)


class DocumentStream:
    """``caches=(qwen, wan)`` fills image elements that name a ``source`` from the visual caches."""

    def __init__(self, root, seed=0, rank=0, world=1, block_rows=4, epochs=1, caches=None):
        self.catalog = Catalog(root)
        self.caches = caches
        self.block_rows, self.rank, self.world, self.epochs = block_rows, rank, world, epochs
        self.blocks = -(-len(self.catalog) // block_rows)
        self.signature = dict(snapshot=self.catalog.snapshot, seed=seed, epoch=0, rank=rank)
        self.seed = seed
        self.cursor = dict(epoch=0, block=rank, row=0)

    def _doc_index(self):
        c = self.cursor
        block = permute(c["block"], self.blocks, self.seed, c["epoch"])
        return block * self.block_rows + c["row"]

    def peek(self):
        while self.cursor["epoch"] < self.epochs:
            if self.cursor["block"] >= self.blocks:
                self.cursor = dict(epoch=self.cursor["epoch"] + 1, block=self.rank, row=0)
                self.signature["epoch"] = self.cursor["epoch"]
                continue
            index = self._doc_index()
            if self.cursor["row"] >= self.block_rows or index >= len(self.catalog):
                self.cursor = dict(epoch=self.cursor["epoch"], block=self.cursor["block"] + self.world, row=0)
                continue
            row = self.catalog.rows[index]
            if self.caches is not None:
                from .cache import attach_cached
                for element in row["elements"]:
                    attach_cached(element, *self.caches)
            return row
        return None

    def advance(self):
        self.cursor = dict(self.cursor, row=self.cursor["row"] + 1)

    def state_dict(self):
        return dict(cursor=dict(self.cursor), signature=dict(self.signature))

    def load_state_dict(self, state):
        saved = dict(state["signature"])
        if {k: saved[k] for k in ("snapshot", "seed", "rank")} != {k: self.signature[k] for k in ("snapshot", "seed", "rank")}:
            raise ValueError("document stream signature differs on resume")
        self.cursor = dict(state["cursor"])
        self.signature["epoch"] = self.cursor["epoch"]

    def close(self):
        pass
