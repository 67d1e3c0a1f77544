"""The DP-sharded, exactly-resumable document stream over a corpus source.

* ``permute``: a constant-memory Feistel bijection over block indices keyed by (seed, epoch), so
  shuffling needs no index table.
* ``DocumentStream``: walks shuffled blocks of ``block_rows`` rows of a source
  (``data.catalog.open_source``: Parquet directory, JSONL file or YAML mixture), assigning blocks
  to DP ranks round-robin. Its cursor ``{epoch, block, row}`` plus a signature (source identity,
  seed, rank) is the resumable state; a resumed stream must present the same signature.
* Preparation runs ahead: a thread pool turns the next ``lookahead`` rows into packer documents
  (reading the row, tokenizing raw text with the batch-capable ``encode``, loading visuals through
  ``visual``), in cursor order. ``peek()`` waits only for the document at the cursor. Documents
  are a pure function of their cursor position, so resuming rebuilds the same window.
Rows that already carry ``elements`` (pre-tokenized) pass through; rows with ``segments`` go
through the chat templating (``data.chat.row_document``). Reference ``data/stream.py:19-256``.
"""

from __future__ import annotations

import hashlib
from collections import deque
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .catalog import open_source


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


def _as_document(row, encode, visual, caches):
    if "elements" in row:
        doc = dict(row)
        doc["elements"] = [dict(e) for e in row["elements"]]
        for e in doc["elements"]:
            if e["type"] == "text":
                if "input_ids" not in e:
                    e["input_ids"] = encode(e.pop("text"))
                e["input_ids"] = np.asarray(e["input_ids"], dtype=np.int64)
            elif visual is not None and "features" not in e:
                e.update(visual(e, row))
    else:
        if encode is None:
            raise ValueError("raw text rows need a tokenizer (encode)")
        from .chat import row_document
        doc = row_document(row, encode, visual)
        for e in doc["elements"]:
            if e["type"] == "text":
                e["input_ids"] = np.asarray(e["input_ids"], dtype=np.int64)
    if caches is not None:
        from .cache import attach_cached
        for element in doc["elements"]:
            attach_cached(element, *caches)
    return doc


class DocumentStream:
    """``encode(text) -> ids`` tokenizes raw text; ``visual(segment, row) -> dict`` loads a visual
    (pixels or cached features); ``caches=(qwen, wan)`` fills image elements that name a
    ``source`` from the visual caches; ``workers`` threads prepare ``lookahead`` rows ahead."""

    def __init__(self, root, seed=0, rank=0, world=1, block_rows=4, epochs=1, caches=None, encode=None, visual=None,
                 workers=4, lookahead=32, cache_bytes=256 << 20):
        self.source = open_source(root, cache_bytes)
        self.caches, self.encode, self.visual = caches, encode, visual
        self.block_rows, self.rank, self.world, self.epochs = block_rows, rank, world, epochs
        self.blocks = -(-len(self.source) // block_rows)
        self.snapshot = self.source.identity
        self.signature = dict(snapshot=self.snapshot, seed=seed, epoch=0, rank=rank)
        self.seed = seed
        self.cursor = dict(epoch=0, block=rank, row=0)
        self.lookahead = max(1, lookahead)
        self.pool = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="docstream") if workers else None
        self.window = deque()     # (cursor, future or document) in order, starting at self.cursor
        self.stats = dict(prepared=0, waited_seconds=0.0)

    # ---- cursor walk --------------------------------------------------------------------------
    def _normalize(self, cursor):
        """The first cursor at or after ``cursor`` that names a row, or None at the end."""
        c = dict(cursor)
        while c["epoch"] < self.epochs:
            if c["block"] >= self.blocks:
                c = dict(epoch=c["epoch"] + 1, block=self.rank, row=0)
                continue
            index = permute(c["block"], self.blocks, self.seed, c["epoch"]) * self.block_rows + c["row"]
            if c["row"] >= self.block_rows or index >= len(self.source):
                c = dict(epoch=c["epoch"], block=c["block"] + self.world, row=0)
                continue
            c["index"] = index
            return c
        return None

    def _successor(self, cursor):
        return self._normalize(dict(epoch=cursor["epoch"], block=cursor["block"], row=cursor["row"] + 1))

    def _prepare(self, index):
        return _as_document(self.source.read(index), self.encode, self.visual, self.caches)

    def _fill(self):
        tail = self.window[-1][0] if self.window else None
        nxt = self._normalize(self.cursor) if tail is None else self._successor(tail)
        while nxt is not None and len(self.window) < self.lookahead:
            job = self.pool.submit(self._prepare, nxt["index"]) if self.pool else None
            self.window.append((nxt, job))
            nxt = self._successor(nxt)

    # ---- stream API ---------------------------------------------------------------------------
    def peek(self):
        if not self.window:
            self._fill()
        if not self.window:
            return None
        cursor, job = self.window[0]
        self.cursor = {k: cursor[k] for k in ("epoch", "block", "row")}
        self.signature["epoch"] = cursor["epoch"]
        if job is None:
            doc = self._prepare(cursor["index"])
            self.window[0] = (cursor, _Ready(doc))
            return doc
        if not job.done():
            import time
            t0 = time.perf_counter()
            doc = job.result()
            self.stats["waited_seconds"] += time.perf_counter() - t0
            return doc
        return job.result()

    def advance(self):
        if not self.window:
            self.peek()
        if self.window:
            cursor, _ = self.window.popleft()
            self.stats["prepared"] += 1
            nxt = self._successor(cursor)
            self.cursor = ({k: nxt[k] for k in ("epoch", "block", "row")} if nxt is not None
                           else dict(epoch=self.epochs, block=self.rank, row=0))
            self._fill()

    def state_dict(self):
        return dict(cursor=dict(self.cursor), signature=dict(self.signature))

    def load_state_dict(self, state):
        saved = dict(state["signature"])
        keys = ("snapshot", "seed", "rank")
        if {k: saved[k] for k in keys} != {k: self.signature[k] for k in keys}:
            raise ValueError("document stream signature differs on resume")
        for _, job in self.window:
            if hasattr(job, "cancel"):
                job.cancel()
        self.window.clear()
        self.cursor = dict(state["cursor"])
        self.signature["epoch"] = self.cursor["epoch"]

    def close(self):
        for _, job in self.window:
            if hasattr(job, "cancel"):
                job.cancel()
        self.window.clear()
        if self.pool is not None:
            self.pool.shutdown(wait=False, cancel_futures=True)
        self.source.close()


class _Ready:
    """A finished preparation (the synchronous path without a thread pool)."""

    def __init__(self, doc):
        self.doc = doc

    def done(self):
        return True

    def result(self):
        return self.doc
