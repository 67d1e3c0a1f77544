"""CUDA graphs of the renderer's forward + backward, one per DiT micro-batch geometry.

The Wan DiT runs 30 blocks over a few thousand tokens: its kernels are short (a 2048-row GEMM
takes microseconds), so issuing them from Python leaves the GPU waiting for the host. A graph
replays the whole chunk (forward, flow-matching loss, backward into ``main_grad`` and into the
CQ-condition leaf) with one launch.

``RendererGraphs.run(model, leaf, bound, factor)`` is the graphed form of
``loss = model.renderer(leaf, bound); (loss * factor).backward()`` and returns ``(loss, leaf
gradient)`` (both valid until the next replay of the same graph). A geometry is keyed by every
non-tensor value of ``bound`` and the shape / dtype / stride of every tensor in it. The first
sighting of a key runs eagerly (the warm-up every capture needs: lazily created device state,
library workspaces); the second captures and replays; later sightings copy their inputs into the
captured tensors and replay. What the host does during the backward is kept in step with the
replays:

* parameter readiness marks for the distributed optimizer (``_mark``) are recorded during the
  capture and issued again after every replay, so the bucket reduce-scatters still start;
* kernel launches counted by the extension during the capture are added per replay, so
  ``_ext.launches()`` counts executed kernels.

Graphs are used where the captured work is position independent: CUDA, no activation recompute
inside the DiT, and the Wan renderer. At TP > 1 (``CQB_GRAPHS_TP=0`` keeps it eager) the fused TP kernels
are captured with the rest: they read their call epochs from device counters, so every replay
takes fresh epochs and parity buffers (``parallel.symmetric``). ``CQB_GRAPHS_TP_NCCL=1`` routes the
captured TP linears through NCCL and the plain GEMM instead (``parallel.symmetric.suspended``; the
NCCL collectives are captured). ``CQB_GRAPHS=0`` turns graphs off.
"""

from __future__ import annotations

import os
from collections import OrderedDict
from dataclasses import fields, is_dataclass
from types import SimpleNamespace

import torch

from ..ops import _ext


def _flatten(value, tensors):
    """A hashable spec of ``value`` with each tensor replaced by its slot in ``tensors``."""
    if isinstance(value, torch.Tensor):
        tensors.append(value)
        return ("T", len(tensors) - 1, tuple(value.shape), str(value.dtype), tuple(value.stride()),
                value.device.type)
    if isinstance(value, SimpleNamespace):
        return ("NS", tuple((k, _flatten(v, tensors)) for k, v in sorted(vars(value).items())))
    if is_dataclass(value) and not isinstance(value, type):
        return ("DC", type(value), tuple((f.name, _flatten(getattr(value, f.name), tensors)) for f in fields(value)))
    if isinstance(value, (list, tuple)):
        return ("L" if isinstance(value, list) else "U", tuple(_flatten(v, tensors) for v in value))
    hash(value)
    return ("V", value)


def _rebuild(spec, tensors):
    kind = spec[0]
    if kind == "T":
        return tensors[spec[1]]
    if kind == "NS":
        return SimpleNamespace(**{k: _rebuild(v, tensors) for k, v in spec[1]})
    if kind == "DC":
        values = {name: _rebuild(v, tensors) for name, v in spec[2]}
        return spec[1](**values)
    if kind in ("L", "U"):
        items = [_rebuild(v, tensors) for v in spec[1]]
        return items if kind == "L" else tuple(items)
    return spec[1]


def graphs_enabled(cfg, device, tp):
    if os.environ.get("CQB_GRAPHS", "1") == "0":
        return False
    if tp > 1 and os.environ.get("CQB_GRAPHS_TP", "1") == "0":
        return False
    return (torch.device(device).type == "cuda" and cfg.renderer == "wan"
            and not getattr(cfg, "checkpoint_dit", 0) and not getattr(cfg, "checkpoint_dit_layers", 0))


class _Entry:
    def __init__(self):
        self.seen = 0
        self.graph = None
        self.inputs = None       # static copies of the bound tensors
        self.leaf = None         # static leaf (requires grad)
        self.factor = None       # static loss factor
        self.loss = None
        self.marks = []
        self.launches = 0


class RendererGraphs:
    def __init__(self, optimizer=None, capacity=4, capture_after=1, max_tokens=16384):
        """``capture_after``: eager sightings of a geometry before it is captured. Chunks of more
        than ``max_tokens`` DiT tokens run eagerly: a graph keeps its activations in its own memory
        pool between replays, which the backbone backward could otherwise reuse, and such chunks
        are long enough that launching from the host does not starve the GPU."""
        self.optimizer = optimizer
        self.capacity = capacity
        self.capture_after = capture_after
        self.max_tokens = max_tokens
        self.entries: OrderedDict = OrderedDict()
        self.pool = None
        self.replays = 0

    def release(self):
        """Drop every captured graph and its memory pool. Graphs that captured NCCL calls must be
        released before the process group is destroyed, or the teardown waits on them."""
        self.entries.clear()
        self.pool = None
        if torch.cuda.is_available():
            torch.cuda.synchronize()

    def _key(self, leaf, bound):
        tensors = []
        spec = _flatten(bound, tensors)
        return (spec, tuple(leaf.shape), str(leaf.dtype), torch.is_grad_enabled()), tensors

    def run(self, model, leaf, bound, factor):
        from ..parallel import state as ps, symmetric
        if self.optimizer is not None and hasattr(self.optimizer, "wait_params"):
            # pending DP parameter all-gathers: the stream waits for them here, outside any capture
            # (their forward pre-hooks would otherwise wait on uncaptured work inside it)
            self.optimizer.wait_params()
        if ps.tp_size() > 1 and os.environ.get("CQB_GRAPHS_TP_NCCL") == "1":
            with symmetric.suspended():
                return self._run(model, leaf, bound, factor)
        return self._run(model, leaf, bound, factor)

    def _run(self, model, leaf, bound, factor):
        lengths = getattr(getattr(bound, "generation", None), "lengths", ())
        if sum(lengths) > self.max_tokens:
            return self._eager(model, leaf, bound, factor)
        key, tensors = self._key(leaf, bound)
        entry = self.entries.get(key)
        if entry is None:
            entry = self.entries[key] = _Entry()
            while len(self.entries) > self.capacity:
                self.entries.popitem(last=False)
        self.entries.move_to_end(key)
        entry.seen += 1
        if entry.graph is None and entry.seen <= self.capture_after:
            return self._eager(model, leaf, bound, factor)
        if entry.graph is None:
            self._capture(entry, model, key, leaf, tensors, factor)
        for dst, src in zip(entry.inputs, tensors):
            dst.copy_(src, non_blocking=True)
        with torch.no_grad():
            entry.leaf.copy_(leaf)
            entry.factor.fill_(float(factor))
        entry.graph.replay()
        self.replays += 1
        _ext.add_graph_launches(entry.launches)
        if self.optimizer is not None:
            for p in entry.marks:
                self.optimizer._mark(p)
        return entry.loss, entry.leaf.grad

    @staticmethod
    def _eager(model, leaf, bound, factor):
        loss = model.renderer(leaf, bound)
        (loss * factor).backward()
        return loss.detach(), leaf.grad

    def _capture(self, entry, model, key, leaf, tensors, factor):
        entry.inputs = [t.detach().clone() for t in tensors]
        static_bound = _rebuild(key[0], entry.inputs)
        entry.leaf = leaf.detach().clone().requires_grad_(leaf.requires_grad)
        entry.factor = torch.full((), float(factor), dtype=torch.float32, device=leaf.device)
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        before = _ext.launches()
        if self.optimizer is not None:
            self.optimizer.start_recording()
        try:
            with torch.cuda.graph(graph, pool=self.pool):
                loss = model.renderer(entry.leaf, static_bound)
                (loss * entry.factor).backward()
                entry.loss = loss.detach()
        finally:
            if self.optimizer is not None:
                entry.marks = self.optimizer.stop_recording()
        entry.launches = _ext.launches() - before
        # the captured kernels did not run: their host-side count is added back per replay
        _ext.add_graph_launches(-entry.launches)
        entry.graph = graph
