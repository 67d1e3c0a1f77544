"""Learning-rate schedule: linear warmup, then constant or cosine decay to ``min_lr``
(reference ``training/train.py:140-147``)."""

from __future__ import annotations

import math


def learning_rate(step, lr, warmup=0, total=0, style="cosine", min_lr=None):
    min_lr = lr * 0.1 if min_lr is None else min_lr
    if warmup and step < warmup:
        return lr * (step + 1) / warmup
    if style == "constant" or not total or total <= warmup:
        return lr
    progress = min(1.0, (step - warmup) / max(1, total - warmup))
    return min_lr + 0.5 * (lr - min_lr) * (1 + math.cos(math.pi * progress))
