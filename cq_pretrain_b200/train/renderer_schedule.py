"""Chunked renderer backward: bound DiT activation memory, backpropagate the backbone once.

The DiT runs over CPU-planned chunks of generation targets on *detached* leaves of the CQ
conditions, one backward per chunk; the leaf gradients are copied into one buffer; finally a
single multi-root backward of ``(loss, conditions <- gradient)`` runs through the backbone
(joining text CE and all CQ gradients). Only the last chunk may trigger renderer bucket
reductions (reference ``training/renderer_schedule.py:34-77``).
"""

from __future__ import annotations

from contextlib import nullcontext
from types import SimpleNamespace

import torch


class _Whole:
    """The whole generation layout as one DiT chunk."""

    start = 0

    def __init__(self, batch):
        self.stop = batch.generation.count

    @staticmethod
    def bind(batch):
        return SimpleNamespace(generation=batch.generation, latents=batch.latents, noise=batch.noise,
                               times=batch.times)


def backward_deferred_renderer(model, batch, losses, backward_scale=1.0, optimizer=None, *, image_factor,
                               timer=None, graphs=None):
    """``timer`` (``utils.observe.PhaseTimer``, optional) times each chunk's DiT forward and
    backward as ``renderer_forward`` / ``renderer_backward`` and the backbone pass as ``backward``.
    ``graphs`` (``train.graphed.RendererGraphs``, optional) runs each chunk's forward + backward as
    a CUDA-graph replay; with graphs, a batch without planned micro-batches is one chunk."""
    from ..utils.observe import phase
    conditions = losses.pop("image_conditions")
    parts = batch.generation.microbatches
    if not parts and graphs is not None:
        parts = (_Whole(batch),)
    if not parts:
        raise ValueError("missing CPU-planned DiT micro-batches")
    gradient = torch.empty_like(conditions) if conditions.requires_grad else None
    image_loss = torch.zeros((), device=conditions.device, dtype=torch.float32)
    for index, part in enumerate(parts):
        leaf = conditions[part.start:part.stop].detach().requires_grad_(gradient is not None)
        last = index + 1 == len(parts)
        context = optimizer.suspend_readiness() if (optimizer is not None and not last) else nullcontext()
        with context:
            if graphs is not None:
                with phase(timer, "renderer_backward"):
                    chunk_loss, leaf_grad = graphs.run(model, leaf, part.bind(batch), image_factor * backward_scale)
            else:
                with phase(timer, "renderer_forward"):
                    chunk_loss = model.renderer(leaf, part.bind(batch))
                with phase(timer, "renderer_backward"):
                    (chunk_loss * (image_factor * backward_scale)).backward()
                leaf_grad = leaf.grad
        image_loss.add_(chunk_loss.detach().float())
        if gradient is not None:
            if leaf_grad is None:
                raise RuntimeError("renderer did not propagate its CQ gradient")
            gradient[part.start:part.stop].copy_(leaf_grad)
        del chunk_loss, leaf, leaf_grad
    roots, upstream = [losses["loss"] * backward_scale], [None]
    if gradient is not None:
        roots.append(conditions)
        upstream.append(gradient)
    with phase(timer, "backward"):
        torch.autograd.backward(roots, upstream)
    losses["loss"] = losses["loss"].detach() + image_loss * image_factor
    losses["text_loss"] = losses["text_loss"].detach()
    losses["image_loss"] = image_loss
    return losses
