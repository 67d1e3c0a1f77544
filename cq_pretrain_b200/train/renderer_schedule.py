"""Chunked renderer backward: bound DiT activation memory, backpropagate the backbone once.

The DiT runs over CPU-planned chunks of generation targets on *detached* leaves of the CQ
conditions, one backward per chunk; the leaf gradients are copied into one buffer; finally a
single multi-root backward of ``(loss, conditions <- gradient)`` runs through the backbone
(joining text CE and all CQ gradients). Only the last chunk may trigger renderer bucket
reductions (reference ``training/renderer_schedule.py:34-77``).
"""

from __future__ import annotations

from contextlib import nullcontext

import torch


def backward_deferred_renderer(model, batch, losses, backward_scale=1.0, optimizer=None, *, image_factor,
                               timer=None):
    """``timer`` (``utils.observe.PhaseTimer``, optional) counts each chunk's DiT forward as
    forward time and the backward passes as backward time."""
    from ..utils.observe import phase
    conditions = losses.pop("image_conditions")
    parts = batch.generation.microbatches
    if not parts:
        raise ValueError("missing CPU-planned DiT micro-batches")
    gradient = torch.empty_like(conditions) if conditions.requires_grad else None
    image_loss = torch.zeros((), device=conditions.device, dtype=torch.float32)
    for index, part in enumerate(parts):
        leaf = conditions[part.start:part.stop].detach().requires_grad_(gradient is not None)
        last = index + 1 == len(parts)
        context = optimizer.suspend_readiness() if (optimizer is not None and not last) else nullcontext()
        with context:
            with phase(timer, "renderer_forward"):
                chunk_loss = model.renderer(leaf, part.bind(batch))
            with phase(timer, "renderer_backward"):
                (chunk_loss * (image_factor * backward_scale)).backward()
        image_loss.add_(chunk_loss.detach().float())
        if gradient is not None:
            if leaf.grad is None:
                raise RuntimeError("renderer did not propagate its CQ gradient")
            gradient[part.start:part.stop].copy_(leaf.grad)
        del chunk_loss, leaf
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
