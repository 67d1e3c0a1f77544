"""Bounded host→device prefetch on a side CUDA stream, with acknowledged-only consumption.

``DeviceLoader(host_loader, preparer, prefetch)`` keeps up to ``prefetch`` packs already copied to
the GPU: each is prepared (flow randomness + pinned-memory ``non_blocking`` copies) on a
dedicated stream and gets a CUDA event. ``next()`` hands out the oldest item without waiting on
the GPU; ``acquire(item)`` makes the current stream wait for the item's event right before its
forward and marks every device tensor as used on that stream (``record_stream``), so the caching
allocator never recycles a tensor the side stream allocated while compute still reads it. The
pinned host batch stays referenced until its copies completed.

The cursor that a checkpoint stores is the host loader's **acknowledged** state: a pack counts
as consumed only after ``acknowledge(receipt)``, which the trainer calls after a successful
optimizer update (reference ``data/device.py:9-173``, ``data/packing.py:434-477``).
``prefetch=0`` is the synchronous control (prepare on the current stream when asked).
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, fields, is_dataclass

import torch


def tensors(value, seen=None):
    """Every tensor reachable through dataclasses, dicts, lists and tuples (each once)."""
    seen = set() if seen is None else seen
    if id(value) in seen:
        return
    seen.add(id(value))
    if isinstance(value, torch.Tensor):
        yield value
    elif is_dataclass(value) and not isinstance(value, type):
        for f in fields(value):
            yield from tensors(getattr(value, f.name), seen)
    elif isinstance(value, dict):
        for v in value.values():
            yield from tensors(v, seen)
    elif isinstance(value, (list, tuple)):
        for v in value:
            yield from tensors(v, seen)


@dataclass
class DeviceItem:
    batch: object
    receipt: dict
    ready: object          # torch.cuda.Event or None
    host: object           # keeps the pinned source alive until the copy finished
    prepare_seconds: float

    def __iter__(self):
        return iter((self.batch, self.receipt))


class DeviceLoader:
    def __init__(self, host_loader, preparer, prefetch=2):
        if prefetch < 0:
            raise ValueError("device prefetch must be >= 0 (0 is the synchronous control)")
        self.host, self.preparer, self.prefetch = host_loader, preparer, prefetch
        device = torch.device(preparer.device)
        self.cuda = device.type == "cuda"
        self.stream = torch.cuda.Stream(device=device) if self.cuda and prefetch else None
        self.pending = deque()
        self.exhausted = False
        self.stats = dict(host_wait_seconds=0.0, prepare_seconds=0.0, acquired=0, not_ready_on_acquire=0,
                          max_queued=0)

    def _prepare(self, host_batch, receipt):
        start = time.perf_counter()
        if self.stream is not None:
            # the side stream must not start copying into memory the main stream still uses
            self.stream.wait_stream(torch.cuda.current_stream(self.stream.device))
            with torch.cuda.stream(self.stream):
                batch = self.preparer(host_batch, receipt, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(self.stream)
        else:
            batch = self.preparer(host_batch, receipt, non_blocking=self.cuda)
            ready = None
        seconds = time.perf_counter() - start
        self.stats["prepare_seconds"] += seconds
        return DeviceItem(batch, receipt, ready, host_batch, seconds)

    def _fill(self):
        while not self.exhausted and len(self.pending) < max(1, self.prefetch):
            start = time.perf_counter()
            got = self.host.next()
            self.stats["host_wait_seconds"] += time.perf_counter() - start
            if got is None:
                self.exhausted = True
                break
            self.pending.append(self._prepare(*got))
            self.stats["max_queued"] = max(self.stats["max_queued"], len(self.pending))

    def next(self):
        """The next prepared item, or ``None`` when the host stream is exhausted."""
        self._fill()
        if not self.pending:
            return None
        item = self.pending.popleft()
        self._fill()   # start preparing the following packs while this one computes
        return item

    def acquire(self, item):
        """Order the current stream after ``item``'s copies; returns ``(batch, receipt)``."""
        if item.ready is not None:
            if not item.ready.query():
                self.stats["not_ready_on_acquire"] += 1
            stream = torch.cuda.current_stream(self.stream.device)
            stream.wait_event(item.ready)
            for t in tensors(item.batch):
                if t.is_cuda:
                    t.record_stream(stream)
        item.host = None
        self.stats["acquired"] += 1
        return item.batch, item.receipt

    def acknowledge(self, receipt):
        self.host.acknowledge(receipt)

    def state_dict(self):
        return self.host.state_dict()

    def close(self):
        self.pending.clear()
        if hasattr(self.host, "close"):
            self.host.close()
