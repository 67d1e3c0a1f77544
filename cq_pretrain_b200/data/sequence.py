"""Token layouts of one visual element inside a packed sequence.

An image is ``[BOI, n merged visual tokens, EOI]``; the visual tokens share one visibility
rank (``sigma``) so they read each other bidirectionally, and their MRoPE coordinates are
(t, h, w) on the merged grid (reference ``data/sequence.py:53-61``). A video is a run of time
blocks, each ``[time text, BOI, h*w tokens, EOI]``; tokens of one block share a rank, so
visibility is bidirectional inside a block and causal across blocks (reference
``data/sequence.py:11-50``). Timestamps are written as plain marker tokens here because the
synthetic path has no tokenizer; the layout rules are the same.
"""

from __future__ import annotations

import numpy as np


def merged_grid(grid):
    """Qwen vision grid (t, h, w) in 16-pixel patches -> merged token grid (t, h/2, w/2)."""
    t, h, w = grid
    return t, h // 2, w // 2


def image_sequence(grid, tokens):
    _, h, w = merged_grid(grid)
    n = h * w
    ids = np.full(n + 2, tokens["image"], dtype=np.int64)
    ids[0], ids[-1] = tokens["boi"], tokens["eoi"]
    sigma = np.arange(n + 2, dtype=np.int64)
    sigma[1:-1] = 1
    positions = np.zeros((3, n + 2), dtype=np.float32)
    local = np.arange(n)
    positions[0, 1:-1] = 1
    positions[1, 1:-1] = 1 + local // w
    positions[2, 1:-1] = 1 + local % w
    positions[:, -1] = 1 + max(h, w)
    # BOI is a supervised structural target; corpus text carries the rest.
    return dict(ids=ids, visual=np.arange(1, n + 1), sigma=sigma, positions=positions,
                text_indices=np.array([0], dtype=np.int64))


def video_sequence(grid, tokens, timestamps=None):
    """Time blocks of a video: a marker token, BOI, the block's merged tokens, EOI."""
    t, h, w = merged_grid(grid)
    block = h * w
    per = block + 3
    ids = np.empty(t * per, dtype=np.int64)
    sigma = np.arange(t * per, dtype=np.int64)
    positions = np.zeros((3, t * per), dtype=np.float32)
    visual = []
    cursor = 0
    local = np.arange(block)
    for b in range(t):
        base = b * per
        ids[base] = tokens.get("time", tokens["boi"])
        ids[base + 1] = tokens["boi"]
        ids[base + 2: base + 2 + block] = tokens["image"]
        ids[base + 2 + block] = tokens["eoi"]
        positions[:, base] = cursor
        positions[:, base + 1] = cursor + 1
        cursor += 2
        idx = np.arange(base + 2, base + 2 + block)
        sigma[idx] = base + 2
        positions[0, idx] = cursor
        positions[1, idx] = cursor + local // w
        positions[2, idx] = cursor + local % w
        cursor += max(h, w)
        positions[:, base + 2 + block] = cursor
        cursor += 1
        visual.append(idx)
    return dict(ids=ids, visual=np.concatenate(visual), sigma=sigma, positions=positions,
                text_indices=np.empty(0, dtype=np.int64))
