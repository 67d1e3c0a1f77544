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


# ---- MOSS-Image-Base renderer (legacy) ----------------------------------------------------------
def moss_rope(height, width, text_length, head_dim, base=10000.0):
    """Four-axis RoPE of one packed ``[image tokens, conditions]`` stream (rotate-half layout).

    Axis coordinates per row: image token (y, x) -> (0, text_length, y - (h-1)/2, x - (w-1)/2);
    condition j -> (0, j, 0, 0). Each axis owns ``head_dim / 8`` frequencies
    ``base^(-i / (head_dim / 8))``; phases are fp32 (the pretrained MOSS convention) and cos / sin
    are duplicated over the two halves -> ``[h*w + text_length, head_dim]`` each.
    """
    n = head_dim // 8
    bands = 1.0 / (base ** (torch.arange(n, dtype=torch.float32) / n))
    ys, xs = torch.meshgrid(torch.arange(height, dtype=torch.float32), torch.arange(width, dtype=torch.float32),
                            indexing="ij")
    image = torch.stack((torch.zeros_like(ys), torch.full_like(ys, float(text_length)),
                         ys - (height - 1) / 2, xs - (width - 1) / 2), -1).reshape(-1, 4)
    text = torch.zeros(text_length, 4)
    text[:, 1] = torch.arange(text_length, dtype=torch.float32)
    phase = (torch.cat((image, text))[:, :, None] * bands).reshape(-1, 4 * n)
    return torch.cat((phase.cos(), phase.cos()), -1), torch.cat((phase.sin(), phase.sin()), -1)


@dataclass
class MossGenerationInputs(Movable):
    """Packed MOSS streams: per target ``[h*w noisy latent tokens, q conditions]`` (reference
    ``data/generation.py:49-136``). ``video_indices`` / ``text_indices`` are the rows of the
    packed stream that hold latent tokens / conditions; ``sample_indices`` maps every packed row,
    ``video_sample_indices`` every latent token, to its target."""

    grids: tuple                        # (h, w) latent grid per target (16 pixels per token)
    lengths: tuple                      # latent tokens per target
    query_counts: tuple                 # conditions per target
    ends: tuple                         # cumulative packed rows
    text_ends: tuple                    # cumulative conditions
    video_ends: tuple                   # cumulative latent tokens
    video_indices: torch.Tensor         # [sum L] packed row of each latent token
    text_indices: torch.Tensor          # [sum q] packed row of each condition
    sample_indices: torch.Tensor        # [rows] target of each packed row
    video_sample_indices: torch.Tensor  # [sum L] target of each latent token
    loss_weights: torch.Tensor          # [sum L] 1 / (targets * tokens of that target)
    cos: torch.Tensor                   # [rows, head_dim]
    sin: torch.Tensor
    time_features: torch.Tensor         # [n, 256]
    microbatches: tuple = ()

    @property
    def count(self) -> int:
        return len(self.lengths)

    @property
    def video_rows(self):
        return self.video_indices

    @classmethod
    def prepare(cls, grids, query_counts, head_dim, token_budget=0, max_images=0):
        grids = tuple((int(h), int(w)) for h, w in grids)
        counts = tuple(int(q) for q in query_counts)
        if not grids or min(counts, default=0) < 1:
            raise ValueError("MOSS layouts need targets with at least one condition each")
        lengths = tuple(h * w for h, w in grids)
        video, text, samples, cos, sin, ends, cursor = [], [], [], [], [], [], 0
        for i, ((h, w), n, q) in enumerate(zip(grids, lengths, counts)):
            video.append(torch.arange(cursor, cursor + n))
            text.append(torch.arange(cursor + n, cursor + n + q))
            samples.append(torch.full((n + q,), i, dtype=torch.long))
            c, s = moss_rope(h, w, q, head_dim)
            cos.append(c)
            sin.append(s)
            cursor += n + q
            ends.append(cursor)
        out = cls(grids, lengths, counts, tuple(ends), tuple(accumulate(counts)), tuple(accumulate(lengths)),
                  torch.cat(video), torch.cat(text), torch.cat(samples),
                  torch.repeat_interleave(torch.arange(len(grids)), torch.tensor(lengths)),
                  torch.cat([torch.full((n,), 1.0 / (len(grids) * n)) for n in lengths]),
                  torch.cat(cos), torch.cat(sin), torch.zeros(0))
        ranges, start, used = [], 0, 0
        for i, (n, q) in enumerate(zip(lengths, counts)):
            if token_budget and n + q > token_budget:
                raise ValueError(f"target/condition stream needs {n + q} tokens, above the DiT budget {token_budget}")
            if i > start and ((token_budget and used + n + q > token_budget) or (max_images and i - start >= max_images)):
                ranges.append((start, i))
                start, used = i, 0
            used += n + q
        ranges.append((start, len(lengths)))
        if len(ranges) > 1:
            out.microbatches = tuple(MossGenerationSlice.prepare(out, a, b) for a, b in ranges)
        return out


@dataclass
class MossGenerationSlice(Movable):
    """Targets ``[start, stop)`` of a MOSS layout with local indices; ``bind`` returns views."""

    start: int
    stop: int
    latent_start: int
    latent_stop: int
    row_start: int
    row_stop: int
    layout: MossGenerationInputs

    @classmethod
    def prepare(cls, parent: MossGenerationInputs, a: int, b: int):
        r0 = parent.ends[a - 1] if a else 0
        r1 = parent.ends[b - 1]
        l0, l1 = sum(parent.lengths[:a]), sum(parent.lengths[:b])
        t0 = parent.text_ends[a - 1] if a else 0
        t1 = parent.text_ends[b - 1]
        layout = MossGenerationInputs(
            parent.grids[a:b], parent.lengths[a:b], parent.query_counts[a:b],
            tuple(e - r0 for e in parent.ends[a:b]), tuple(e - t0 for e in parent.text_ends[a:b]),
            tuple(accumulate(parent.lengths[a:b])), parent.video_indices[l0:l1] - r0,
            parent.text_indices[t0:t1] - r0, parent.sample_indices[r0:r1] - a,
            parent.video_sample_indices[l0:l1] - a, parent.loss_weights[l0:l1],
            parent.cos[r0:r1], parent.sin[r0:r1], torch.zeros(0))
        return cls(a, b, l0, l1, r0, r1, layout)

    def bind(self, batch):
        layout = replace(self.layout, time_features=batch.generation.time_features[self.start:self.stop])
        return SimpleNamespace(generation=layout, latents=batch.latents[self.latent_start:self.latent_stop],
                               noise=batch.noise[self.latent_start:self.latent_stop],
                               times=batch.times[self.start:self.stop])
