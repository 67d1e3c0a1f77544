"""Packed batch container and its host/device movement.

A batch is one packed sequence (micro-batch 1, as in the reference ``data/batch.py:10-33``):
content token ids, per-position document segments and visibility ranks, MRoPE coordinates,
the supervised text positions, the content spans of visual elements, and (after planning)
a :class:`~cq_pretrain_b200.data.plan.CQPlan`. Tensors move with ``to``/``pin_memory``;
plan and generation metadata move with them.
"""

from __future__ import annotations

from dataclasses import dataclass, fields, replace

import numpy as np
import torch


def _move(value, fn):
    if isinstance(value, torch.Tensor):
        return fn(value)
    if hasattr(value, "_map"):
        return value._map(fn)
    if isinstance(value, tuple) and value and all(isinstance(x, torch.Tensor) for x in value):
        return tuple(fn(x) for x in value)
    if isinstance(value, tuple) and value and all(hasattr(x, "_map") for x in value):
        return tuple(x._map(fn) for x in value)     # e.g. the planned DiT micro-batch layouts
    return value


class Movable:
    """Dataclass mixin: map every tensor (and nested movable) through ``fn``."""

    def _map(self, fn):
        return replace(self, **{f.name: _move(getattr(self, f.name), fn) for f in fields(self)})

    def to(self, device, non_blocking=False):
        return self._map(lambda t: t.to(device, non_blocking=non_blocking))

    def pin_memory(self):
        return self._map(lambda t: t.pin_memory() if t.numel() and t.device.type == "cpu" else t)


@dataclass
class VisionInputs(Movable):
    """Understanding-side visuals: Qwen patch grids and where their merged tokens sit in content.

    ``features`` are merger outputs ``[sum tokens, width]`` (synthetic or from the visual cache);
    ``pixel_values`` are flattened Qwen patches for the online vision tower.
    """

    grid_thw: tuple
    content_indices: torch.Tensor
    features: torch.Tensor | None = None
    pixel_values: torch.Tensor | None = None
    layout: object = None        # VisionLayout for the online tower (when features are not cached)

    @property
    def token_counts(self):
        return tuple(t * (h // 2) * (w // 2) for t, h, w in self.grid_thw)


@dataclass
class EmbeddingPlan(Movable):
    """Sort plan of the backbone's input ids for the embedding backward, built on the host with the
    batch so that the backward needs no device-to-host round trip: ``order`` (row positions sorted
    by id, stable), ``run_ids`` (each distinct id once, ascending), ``seg_start`` (boundaries in
    ``order`` of segments of at most ``seg`` positions that never cross an id) and ``run_seg``
    (first segment of every id, plus the total)."""

    order: torch.Tensor
    run_ids: torch.Tensor
    seg_start: torch.Tensor
    run_seg: torch.Tensor

    @classmethod
    def build(cls, ids, seg=16):
        ids = np.asarray(ids, dtype=np.int64).reshape(-1)
        order = np.argsort(ids, kind="stable")
        run_ids, counts = np.unique(ids[order], return_counts=True)
        pieces = (counts + seg - 1) // seg
        run_seg = np.concatenate(([0], np.cumsum(pieces)))
        run_start = np.concatenate(([0], np.cumsum(counts)[:-1]))
        owner = np.repeat(np.arange(len(counts)), pieces)
        within = np.arange(int(run_seg[-1])) - run_seg[:-1][owner]
        seg_start = np.concatenate((run_start[owner] + within * seg, [len(ids)]))
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64))
        return cls(t(order), t(run_ids), t(seg_start), t(run_seg))


def backbone_ids(batch, text_mask_id, image_mask_id):
    """Input token of every backbone row: the content ids, each query's mask token (image or text
    query) and text-mask tokens on the padding rows."""
    plan = batch.mainline
    ids = batch.ids.reshape(-1)
    qids = torch.where(plan.query_image.to(ids.device), image_mask_id, text_mask_id).to(ids.dtype)
    pad = plan.rows - plan.content_length - plan.queries
    return torch.cat((ids, qids, ids.new_full((pad,), text_mask_id)))


@dataclass
class Batch(Movable):
    ids: torch.Tensor                      # [1, S] content ids (visual placeholders included)
    segments: torch.Tensor                 # [1, S] packed document id, -1 for padding
    sigma: torch.Tensor                    # [1, S] visibility rank; tied inside visual blocks
    positions: torch.Tensor                # [3, S] MRoPE (t, h, w) coordinates
    text_indices: torch.Tensor             # [T] supervised positions; target = ids[0, p]
    image_indices: torch.Tensor            # [n_visual, max_tokens] content positions, -1 padded
    image_queries: torch.Tensor            # [1, S] bool, True on visual content tokens
    vision: VisionInputs | None = None
    generation: object = None              # WanGenerationInputs for generation targets
    generation_image_indices: torch.Tensor | None = None  # visuals that are generation targets
    generation_unconditional: torch.Tensor | None = None  # [n_visual] bool: non-CFG target
    latents: torch.Tensor | None = None    # [sum L, C*4] clean patchified latents of targets
    noise: torch.Tensor | None = None      # [sum L, C*4]
    times: torch.Tensor | None = None      # [n_targets] flow sigma in (0, 1)
    mainline: object = None                # CQPlan
    embed_plan: object = None              # EmbeddingPlan of the backbone input ids (host-built)

    @property
    def length(self) -> int:
        return self.ids.shape[1]

    @property
    def generation_image_count(self) -> int:
        if self.generation_image_indices is None:
            return len(self.image_indices)
        return int(self.generation_image_indices.numel())

    def targets(self) -> torch.Tensor:
        return self.ids.reshape(-1).index_select(0, self.text_indices)
