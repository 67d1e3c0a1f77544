"""Loss composition and data-parallel loss scales.

``loss = text_weight * s_t * text_loss + image_weight * s_i * image_loss`` with defaults 0.05 and
1.0; a missing image loss becomes zero (reference ``training/loss.py:4-12``). The scales make
each objective a *global* average across DP ranks and accumulation micro-batches whose token
and image counts differ: ``s_t = dp * n_text_local / N_text_global`` and likewise for images
(reference ``training/train.py:150-157,610-628``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def compose_losses(outputs, cfg, scales=None):
    text_scale, image_scale = scales if scales is not None else (1.0, 1.0)
    loss = outputs["text_loss"] * (cfg.text_weight * text_scale)
    image = outputs["image_loss"]
    if image is not None:
        loss = loss + image * (cfg.image_weight * image_scale)
    else:
        image = outputs["text_loss"].detach().new_zeros(())
    return dict(outputs, loss=loss, image_loss=image)


def scales_from_counts(local_text, local_images, total_text, total_images, dp_size):
    """``(s_t, s_i)`` of one micro-batch: its share of all supervised text tokens / generation
    images summed over DP ranks and accumulation steps, times the DP size (the DP gradient is
    averaged over ranks). An objective with no global targets gets scale 0."""
    s_t = dp_size * local_text / total_text if total_text else 0.0
    s_i = dp_size * local_images / total_images if total_images else 0.0
    return s_t, s_i


def loss_scales(local_text, local_images, dp_size, group=None, device="cpu"):
    """Return (s_t, s_i) from local counts; all-reduces the counts over ``group`` when DP > 1."""
    counts = torch.tensor([float(local_text), float(local_images)], dtype=torch.float64, device=device)
    if dp_size > 1:
        dist.all_reduce(counts, group=group)
    total_text, total_images = counts.tolist()
    return scales_from_counts(local_text, local_images, total_text, total_images, dp_size)
