"""Packed Wan2.1 generation geometry: latent patches, 3D RoPE, loss weights, DiT micro-batches.

Images are single-frame videos. Each generation target contributes ``T*H*W`` DiT tokens
(latent frames x latent rows/2 x latent cols/2 for the 1x2x2 patch) and is conditioned on its
own CQ visual-query hidden states. Sequence boundaries are cumulative token counts
(``video_ends``/``text_ends``) so attention runs varlen without a padding mask
(reference ``ops/wan_layout.py:9-58``, ``data/generation.py:189-272``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from itertools import accumulate
from types import SimpleNamespace

import torch

from .batch import Movable


def wan_rope(grid, head_dim):
    """3D RoPE angles for a (T, H, W) token grid: widths (d-4*(d//6), 2*(d//6), 2*(d//6)), base 1e4, float64."""
    coords = torch.stack(torch.meshgrid(*(torch.arange(n, dtype=torch.float64) for n in grid), indexing="ij"),
                         -1).reshape(-1, 3)
    sixth = head_dim // 6
    widths = (head_dim - 4 * sixth, 2 * sixth, 2 * sixth)
    angles = torch.cat([coords[:, i, None] * 10000.0 ** (-torch.arange(0, d, 2, dtype=torch.float64) / d)
                        for i, d in enumerate(widths)], -1)
    return angles.cos().float(), angles.sin().float()


def patch_latent(z: torch.Tensor) -> torch.Tensor:
    """[C, T, H, W] latent -> [T*(H/2)*(W/2), C*4] patches in Conv3d (c, ph, pw) order."""
    c, t, h, w = z.shape
    return z.reshape(c, t, h // 2, 2, w // 2, 2).permute(1, 2, 4, 0, 3, 5).reshape(-1, c * 4)


def unpatch_latent(patches: torch.Tensor, grid, channels=16) -> torch.Tensor:
    t, h, w = grid
    return patches.reshape(t, h, w, channels, 2, 2).permute(3, 0, 1, 4, 2, 5).reshape(channels, t, h * 2, w * 2)


def time_features(times: torch.Tensor, freq_dim: int) -> torch.Tensor:
    """Sinusoidal embedding of ``1000 * sigma`` (cos then sin), computed in float64."""
    half = freq_dim // 2
    freqs = 10000.0 ** (-torch.arange(half, dtype=torch.float64) / half)
    phase = (times.double() * 1000)[:, None] * freqs.to(times.device)
    return torch.cat((phase.cos(), phase.sin()), -1).float()


@dataclass
class WanGenerationInputs(Movable):
    grids: tuple                        # (T, H, W) DiT token grid per target
    lengths: tuple                      # DiT tokens per target
    query_counts: tuple                 # CQ conditions per target
    video_ends: tuple                   # cumulative DiT tokens
    text_ends: tuple                    # cumulative conditions
    video_sample_indices: torch.Tensor  # [sum L] target of each DiT token
    condition_indices: torch.Tensor     # [sum q] rows of the flattened [n, max_q] condition block
    loss_weights: torch.Tensor          # [sum L] 1 / (targets * tokens of that target)
    cos: torch.Tensor                   # [sum L, head_dim/2]
    sin: torch.Tensor
    time_features: torch.Tensor         # [n, freq_dim]
    microbatches: tuple = ()            # WanGenerationSlice tuple when the token budget splits targets

    @property
    def count(self) -> int:
        return len(self.lengths)

    @classmethod
    def prepare(cls, grids, query_counts, head_dim, token_budget=0, max_images=0, condition_width=None):
        grids = tuple(tuple(int(x) for x in g) for g in grids)
        counts = tuple(int(q) for q in query_counts)
        lengths = tuple(math.prod(g) for g in grids)
        width = max(counts) if condition_width is None else condition_width
        samples = torch.repeat_interleave(torch.arange(len(grids)), torch.tensor(lengths, dtype=torch.long))
        cond = torch.cat([torch.arange(q) + i * width for i, q in enumerate(counts)]) if counts else torch.zeros(0, dtype=torch.long)
        ropes = [wan_rope(g, head_dim) for g in grids]
        weights = torch.cat([torch.full((n,), 1.0 / (len(grids) * n)) for n in lengths])
        out = cls(grids, lengths, counts, tuple(accumulate(lengths)), tuple(accumulate(counts)), samples, cond, weights,
                  torch.cat([r[0] for r in ropes]), torch.cat([r[1] for r in ropes]), torch.zeros(0))
        ranges, start, used = [], 0, 0
        for i, n in enumerate(lengths):
            if token_budget and n > token_budget:
                raise ValueError(f"visual target needs {n} Wan tokens, above the budget {token_budget}")
            if i > start and ((token_budget and used + n > token_budget) or (max_images and i - start >= max_images)):
                ranges.append((start, i))
                start, used = i, 0
            used += n
        ranges.append((start, len(lengths)))
        if len(ranges) > 1:
            out.microbatches = tuple(WanGenerationSlice.prepare(out, a, b) for a, b in ranges)
        return out


@dataclass
class WanGenerationSlice(Movable):
    """Targets ``[start, stop)`` of a parent layout; ``bind`` returns views, never copies."""

    start: int
    stop: int
    latent_start: int
    latent_stop: int
    layout: WanGenerationInputs

    @classmethod
    def prepare(cls, parent: WanGenerationInputs, a: int, b: int):
        lo, hi = sum(parent.lengths[:a]), sum(parent.lengths[:b])
        counts = parent.query_counts[a:b]
        width = max(parent.query_counts)
        cond = torch.cat([torch.arange(q) + i * width for i, q in enumerate(counts)])
        layout = WanGenerationInputs(parent.grids[a:b], parent.lengths[a:b], counts,
                                     tuple(accumulate(parent.lengths[a:b])), tuple(accumulate(counts)),
                                     parent.video_sample_indices[lo:hi] - a, cond, parent.loss_weights[lo:hi],
                                     parent.cos[lo:hi], parent.sin[lo:hi], torch.zeros(0))
        return cls(a, b, lo, hi, layout)

    def bind(self, batch):
        layout = replace(self.layout, time_features=batch.generation.time_features[self.start:self.stop])
        return SimpleNamespace(generation=layout, latents=batch.latents[self.latent_start:self.latent_stop],
                               noise=batch.noise[self.latent_start:self.latent_stop],
                               times=batch.times[self.start:self.stop])
