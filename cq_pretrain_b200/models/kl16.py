"""KL16 VAE encoder (the MAR / latent-diffusion KL autoencoder) for the legacy renderer's latents.

Reference ``models/vendor/mar/vae.py:161-490`` (encoder half) and ``data/codec.py:14-66``:

* ``conv_in`` (3x3) -> per level ``num_res_blocks`` residual blocks (GroupNorm(32) + SiLU ->
  3x3 conv, twice; 1x1 shortcut when the width changes) with single-head spatial self-attention
  after each block at the attention resolutions, then a stride-2 3x3 downsample on a
  bottom/right zero-padded input (every level but the last) -> middle (block, attention, block)
  -> GroupNorm + SiLU -> ``conv_out`` to ``2 z`` moments;
* ``quant_conv`` (1x1) on the moments; mean / log-variance halves, log-variance clamped to
  [-30, 20]; the codec returns ``(mean * scale, exp(logvar / 2) * scale)`` with scale 0.2325.

Module and parameter names follow the published checkpoint (``encoder.down.{level}.block.{i}``,
``encoder.mid.attn_1``, ``quant_conv`` ...) so its state dict loads strictly.
"""

from __future__ import annotations

from pathlib import Path

import torch
import torch.nn.functional as F
from torch import nn


def _norm(channels):
    return nn.GroupNorm(32, channels, eps=1e-6, affine=True)


class ResBlock(nn.Module):
    def __init__(self, cin, cout):
        super().__init__()
        self.in_channels, self.out_channels = cin, cout
        self.norm1, self.conv1 = _norm(cin), nn.Conv2d(cin, cout, 3, padding=1)
        self.norm2, self.conv2 = _norm(cout), nn.Conv2d(cout, cout, 3, padding=1)
        if cin != cout:
            self.nin_shortcut = nn.Conv2d(cin, cout, 1)

    def forward(self, x):
        h = self.conv1(F.silu(self.norm1(x)))
        h = self.conv2(F.silu(self.norm2(h)))
        return (self.nin_shortcut(x) if self.in_channels != self.out_channels else x) + h


class SpatialAttention(nn.Module):
    def __init__(self, channels):
        super().__init__()
        self.norm = _norm(channels)
        self.q, self.k, self.v = (nn.Conv2d(channels, channels, 1) for _ in range(3))
        self.proj_out = nn.Conv2d(channels, channels, 1)

    def forward(self, x):
        b, c, h, w = x.shape
        y = self.norm(x)
        q, k, v = (conv(y).reshape(b, 1, c, h * w).transpose(-1, -2) for conv in (self.q, self.k, self.v))
        out = F.scaled_dot_product_attention(q, k, v)           # scale c^-1/2, one head over h*w
        return x + self.proj_out(out.transpose(-1, -2).reshape(b, c, h, w))


class Downsample(nn.Module):
    def __init__(self, channels):
        super().__init__()
        self.conv = nn.Conv2d(channels, channels, 3, stride=2)

    def forward(self, x):
        return self.conv(F.pad(x, (0, 1, 0, 1)))


class Encoder(nn.Module):
    def __init__(self, ch=128, ch_mult=(1, 1, 2, 2, 4), num_res_blocks=2, attn_resolutions=(16,), in_channels=3,
                 resolution=256, z_channels=16):
        super().__init__()
        self.num_resolutions, self.num_res_blocks = len(ch_mult), num_res_blocks
        self.conv_in = nn.Conv2d(in_channels, ch, 3, padding=1)
        widths = (1,) + tuple(ch_mult)
        self.down = nn.ModuleList()
        res = resolution
        width = ch
        for level, mult in enumerate(ch_mult):
            stage = nn.Module()
            stage.block, stage.attn = nn.ModuleList(), nn.ModuleList()
            width = ch * widths[level]
            for _ in range(num_res_blocks):
                stage.block.append(ResBlock(width, ch * mult))
                width = ch * mult
                if res in attn_resolutions:
                    stage.attn.append(SpatialAttention(width))
            if level != len(ch_mult) - 1:
                stage.downsample = Downsample(width)
                res //= 2
            self.down.append(stage)
        self.mid = nn.Module()
        self.mid.block_1, self.mid.attn_1, self.mid.block_2 = ResBlock(width, width), SpatialAttention(width), ResBlock(width, width)
        self.norm_out = _norm(width)
        self.conv_out = nn.Conv2d(width, 2 * z_channels, 3, padding=1)

    def forward(self, x):
        h = self.conv_in(x)
        for level, stage in enumerate(self.down):
            for i, block in enumerate(stage.block):
                h = block(h)
                if len(stage.attn):
                    h = stage.attn[i](h)
            if level != self.num_resolutions - 1:
                h = stage.downsample(h)
        h = self.mid.block_2(self.mid.attn_1(self.mid.block_1(h)))
        return self.conv_out(F.silu(self.norm_out(h)))


class FrozenKL16(nn.Module):
    """Frozen KL16 encoder + quant_conv; ``encode`` returns the scaled posterior (mean, std)."""

    def __init__(self, checkpoint=None, dtype=torch.float32, device="cpu", scale=0.2325, chunk=2, z_channels=16):
        super().__init__()
        self.encoder = Encoder(z_channels=z_channels)
        self.quant_conv = nn.Conv2d(2 * z_channels, 2 * z_channels, 1)
        if checkpoint is not None:
            state = torch.load(Path(checkpoint), map_location="cpu", weights_only=True, mmap=True)["model"]
            state = {k: v for k, v in state.items() if k.startswith(("encoder.", "quant_conv."))}
            self.load_state_dict(state, strict=True)
        self.requires_grad_(False).eval().to(device=device, dtype=dtype)
        self.scale, self.chunk, self.dtype = float(scale), int(chunk), dtype

    @torch.no_grad()
    def encode(self, pixels):
        moments = [self.quant_conv(self.encoder(pixels[i:i + self.chunk].to(self.dtype))).float()
                   for i in range(0, len(pixels), self.chunk)]
        mean, logvar = torch.cat(moments).chunk(2, 1)
        return mean * self.scale, logvar.clamp(-30, 20).mul(0.5).exp() * self.scale
