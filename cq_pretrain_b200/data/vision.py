"""Qwen-style native-resolution image/video preprocessing for the understanding tower.

``smart_size`` picks a size whose sides are multiples of 32 (16-pixel patches merged 2x2),
keeps the aspect ratio and lands inside ``[min_pixels, max_pixels]``. ``patchify`` turns frames
``[T, 3, H, W]`` (T padded to a multiple of the temporal patch 2) into rows of
``3*2*16*16`` values ordered so every 4 consecutive rows form one 2x2 merge group, and
``VisionLayout.prepare`` computes, per patch, the 4 bilinear indices/weights into the learned
position grid and the 2-D rotary angles (float64 trig, cast to float32)
(reference ``data/vision.py:26-212``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .batch import Movable

MEAN = (0.5, 0.5, 0.5)
STD = (0.5, 0.5, 0.5)


def smart_size(height, width, min_pixels=65536, max_pixels=1048576, factor=32):
    if max(height, width) > 200 * min(height, width):
        raise ValueError("aspect ratio above 200:1")
    h = max(factor, round(height / factor) * factor)
    w = max(factor, round(width / factor) * factor)
    if h * w > max_pixels:
        beta = math.sqrt(height * width / max_pixels)
        h = max(factor, math.floor(height / beta / factor) * factor)
        w = max(factor, math.floor(width / beta / factor) * factor)
    elif h * w < min_pixels:
        beta = math.sqrt(min_pixels / (height * width))
        h = math.ceil(height * beta / factor) * factor
        w = math.ceil(width * beta / factor) * factor
    return h, w


def patchify(frames, patch=16, temporal=2, merge=2):
    """frames float ``[T, 3, H, W]`` -> (patches ``[t*h*w, 3*temporal*patch*patch]``, grid (t, h, w))."""
    t_frames, c, height, width = frames.shape
    if t_frames % temporal:
        frames = torch.cat((frames, frames[-1:].expand(temporal - t_frames % temporal, -1, -1, -1)))
    t = frames.shape[0] // temporal
    h, w = height // patch, width // patch
    x = frames.reshape(t, temporal, c, h // merge, merge, patch, w // merge, merge, patch)
    x = x.permute(0, 3, 6, 4, 7, 2, 1, 5, 8)   # t, hm, wm, mh, mw, c, temporal, ph, pw
    return x.reshape(t * h * w, c * temporal * patch * patch), (t, h, w)


def preprocess_image(rgb, min_pixels=65536, max_pixels=1048576):
    """uint8 ``[H, W, 3]`` -> (patches, grid). Bicubic resize with PIL, then normalise to [-1, 1]."""
    from PIL import Image
    h, w = smart_size(rgb.shape[0], rgb.shape[1], min_pixels, max_pixels)
    image = Image.fromarray(rgb).resize((w, h), Image.Resampling.BICUBIC)
    x = torch.from_numpy(np.asarray(image, dtype=np.float32) / 255.0).permute(2, 0, 1)
    x = (x - torch.tensor(MEAN)[:, None, None]) / torch.tensor(STD)[:, None, None]
    return patchify(x[None])


@dataclass
class VisionLayout(Movable):
    pixel_values: torch.Tensor   # [patches, 1536]
    pos_indices: torch.Tensor    # [4, patches] indices into the learned position grid
    pos_weights: torch.Tensor    # [4, patches] bilinear weights
    cos: torch.Tensor            # [patches, head_dim/2] 2-D rotary (rows then cols)
    sin: torch.Tensor
    grids: tuple
    lengths: tuple               # patches per frame block (attention is within one image/frame)
    ends: tuple

    @classmethod
    def prepare(cls, pixel_values, grids, num_positions=2304, head_dim=64, merge=2, theta=10000.0):
        side = int(math.isqrt(num_positions))
        inv = theta ** (-torch.arange(0, head_dim // 2, 2, dtype=torch.float64) / (head_dim // 2))
        idx_all, w_all, ang_all, lengths = [], [], [], []
        for t, h, w in grids:
            ys = torch.linspace(0, side - 1, h, dtype=torch.float64)
            xs = torch.linspace(0, side - 1, w, dtype=torch.float64)
            y0, x0 = ys.floor().long(), xs.floor().long()
            y1, x1 = (y0 + 1).clamp(max=side - 1), (x0 + 1).clamp(max=side - 1)
            dy, dx = ys - y0, xs - x0
            # merge order of the patches: (h/2, w/2, 2, 2)
            rows = torch.arange(h).reshape(h // merge, merge)[:, None, :, None].expand(h // merge, w // merge, merge, merge)
            cols = torch.arange(w).reshape(w // merge, merge)[None, :, None, :].expand(h // merge, w // merge, merge, merge)
            r, c = rows.reshape(-1), cols.reshape(-1)
            idx = torch.stack([y0[r] * side + x0[c], y0[r] * side + x1[c], y1[r] * side + x0[c], y1[r] * side + x1[c]])
            wts = torch.stack([(1 - dy[r]) * (1 - dx[c]), (1 - dy[r]) * dx[c], dy[r] * (1 - dx[c]), dy[r] * dx[c]])
            angle = torch.cat((r[:, None].double() * inv, c[:, None].double() * inv), -1)
            idx_all.append(idx.repeat(1, t))
            w_all.append(wts.repeat(1, t).float())
            ang_all.append(angle.repeat(t, 1))
            lengths.extend([h * w] * t)
        angles = torch.cat(ang_all)
        angles = torch.cat((angles, angles), -1)   # rotate-half layout over the full head dim
        ends = tuple(int(x) for x in torch.tensor(lengths).cumsum(0))
        return cls(pixel_values, torch.cat(idx_all, 1), torch.cat(w_all, 1), angles.cos().float(), angles.sin().float(),
                   tuple(grids), tuple(lengths), ends)
