"""Wan2.1 video VAE (causal 3-D convolutional autoencoder, 8x spatial / 4x temporal, 16 latent
channels), written so the published ``Wan2.1_VAE.pth`` state dict loads by name.

Geometry: a video ``[B, 3, 1 + 4k, H, W]`` encodes to ``[B, 16, 1 + k, H/8, W/8]``; the first frame
is encoded on its own (an image is a one-frame video) and later frames in groups of four. Every
temporal convolution is causal (zero or cached frames in front, none behind), so processing the
video group by group with a per-layer cache of the last input frames gives the same result as one
pass over the whole video while holding only one group of activations. The cache entry of a layer
is the last ``CACHE_FRAMES`` frames it saw (fewer at the start); the temporal downsampling stage
caches the last frame of its 2-D output and the temporal upsampling stage marks its first call
(the first latent frame decodes to one frame, each later one to four).

Blocks (channel counts for ``dim = 96``, multipliers 1, 2, 4, 4):
* ``CausalConv3d``: Conv3d whose time padding is all in front (``2 p_t`` frames), space padding
  symmetric.
* ``ChannelRMSNorm``: ``normalize(x, dim=channels) * sqrt(C) * gamma (+ bias)``.
* ``ResidualBlock``: norm, SiLU, 3x3x3 causal conv, norm, SiLU, dropout, 3x3x3 causal conv, plus a
  1x1x1 shortcut when the width changes.
* ``AttentionBlock``: per-frame single-head self-attention over the pixels of the frame, 1x1 conv
  q/k/v and output projection (zero-initialised), residual.
* ``Resample``: 2x nearest-exact spatial upsampling + 3x3 conv halving the width (``upsample2d``),
  plus a (3, 1, 1) causal time conv doubling the frames (``upsample3d``); stride-2 3x3 conv after a
  (0, 1, 0, 1) zero pad (``downsample2d``), plus a stride-2 (3, 1, 1) time conv over the previous
  frame and the new ones (``downsample3d``).
* ``Encoder3d`` / ``Decoder3d`` around a middle (residual, attention, residual), and the 1x1x1
  ``conv1`` (posterior: mean and log-variance) / ``conv2`` (latent -> decoder input).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

CACHE_FRAMES = 2


class CausalConv3d(nn.Conv3d):
    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        pt, ph, pw = self.padding
        self.pads = (pw, pw, ph, ph, 2 * pt, 0)   # F.pad order: w, h, t (front only)
        self.padding = (0, 0, 0)

    def forward(self, x, cache=None):
        pads = list(self.pads)
        if cache is not None and pads[4] > 0:
            x = torch.cat((cache.to(x), x), 2)
            pads[4] = max(0, pads[4] - cache.shape[2])
        return super().forward(F.pad(x, pads))


class ChannelRMSNorm(nn.Module):
    def __init__(self, dim, images=True, bias=False):
        super().__init__()
        shape = (dim, 1, 1) if images else (dim, 1, 1, 1)
        self.scale = dim ** 0.5
        self.gamma = nn.Parameter(torch.ones(shape))
        self.bias = nn.Parameter(torch.zeros(shape)) if bias else None

    def forward(self, x):
        y = F.normalize(x, dim=1) * self.scale * self.gamma
        return y + self.bias if self.bias is not None else y


class _Cache:
    """Per-layer caches of one chunked encode / decode, consumed in call order."""

    def __init__(self):
        self.slots = []
        self.index = 0

    def rewind(self):
        self.index = 0

    def take(self):
        if self.index == len(self.slots):
            self.slots.append(None)
        self.index += 1
        return self.index - 1


def _cached_conv(conv, x, cache):
    """``conv(x)`` continuing the frames the cache holds; the cache then keeps x's last frames."""
    if cache is None:
        return conv(x)
    slot = cache.take()
    prev = cache.slots[slot]
    keep = x[:, :, -CACHE_FRAMES:].clone()
    if keep.shape[2] < CACHE_FRAMES and prev is not None:
        keep = torch.cat((prev[:, :, -1:].to(keep), keep), 2)
    out = conv(x, prev)
    cache.slots[slot] = keep
    return out


class ResidualBlock(nn.Module):
    def __init__(self, in_dim, out_dim, dropout=0.0):
        super().__init__()
        self.residual = nn.Sequential(
            ChannelRMSNorm(in_dim, images=False), nn.SiLU(), CausalConv3d(in_dim, out_dim, 3, padding=1),
            ChannelRMSNorm(out_dim, images=False), nn.SiLU(), nn.Dropout(dropout),
            CausalConv3d(out_dim, out_dim, 3, padding=1))
        self.shortcut = CausalConv3d(in_dim, out_dim, 1) if in_dim != out_dim else nn.Identity()

    def forward(self, x, cache=None):
        h = self.shortcut(x)
        for layer in self.residual:
            x = _cached_conv(layer, x, cache) if isinstance(layer, CausalConv3d) else layer(x)
        return x + h


class AttentionBlock(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.norm = ChannelRMSNorm(dim)
        self.to_qkv = nn.Conv2d(dim, dim * 3, 1)
        self.proj = nn.Conv2d(dim, dim, 1)
        nn.init.zeros_(self.proj.weight)

    def forward(self, x, cache=None):
        b, c, t, h, w = x.shape
        frames = x.permute(0, 2, 1, 3, 4).reshape(b * t, c, h, w)
        qkv = self.to_qkv(self.norm(frames)).reshape(b * t, 3 * c, h * w).transpose(1, 2)
        q, k, v = qkv[:, None].chunk(3, dim=-1)     # [bt, 1 head, pixels, c]
        y = F.scaled_dot_product_attention(q.contiguous(), k.contiguous(), v.contiguous())
        y = self.proj(y[:, 0].transpose(1, 2).reshape(b * t, c, h, w))
        return x + y.reshape(b, t, c, h, w).permute(0, 2, 1, 3, 4)


class _Nearest(nn.Module):
    def forward(self, x):
        return F.interpolate(x.float(), scale_factor=2.0, mode="nearest-exact").to(x.dtype)


class Resample(nn.Module):
    MODES = ("none", "upsample2d", "upsample3d", "downsample2d", "downsample3d")

    def __init__(self, dim, mode):
        super().__init__()
        if mode not in self.MODES:
            raise ValueError(f"unknown resample mode {mode}")
        self.mode = mode
        if mode.startswith("upsample"):
            self.resample = nn.Sequential(_Nearest(), nn.Conv2d(dim, dim // 2, 3, padding=1))
        elif mode.startswith("downsample"):
            self.resample = nn.Sequential(nn.ZeroPad2d((0, 1, 0, 1)), nn.Conv2d(dim, dim, 3, stride=2))
        else:
            self.resample = nn.Identity()
        if mode == "upsample3d":
            self.time_conv = CausalConv3d(dim, dim * 2, (3, 1, 1), padding=(1, 0, 0))
        elif mode == "downsample3d":
            self.time_conv = CausalConv3d(dim, dim, (3, 1, 1), stride=(2, 1, 1), padding=(0, 0, 0))

    def forward(self, x, cache=None):
        b, c, t, h, w = x.shape
        if self.mode == "upsample3d" and cache is not None:
            slot = cache.take()
            prev = cache.slots[slot]
            if prev is None:                     # the first latent frame decodes to one frame
                cache.slots[slot] = "first"
            else:
                keep = x[:, :, -CACHE_FRAMES:].clone()
                if keep.shape[2] < CACHE_FRAMES:
                    front = torch.zeros_like(keep) if isinstance(prev, str) else prev[:, :, -1:].to(keep)
                    keep = torch.cat((front, keep), 2)
                x = self.time_conv(x) if isinstance(prev, str) else self.time_conv(x, prev)
                cache.slots[slot] = keep
                x = x.reshape(b, 2, c, t, h, w).permute(0, 2, 3, 1, 4, 5).reshape(b, c, 2 * t, h, w)
        t = x.shape[2]
        y = self.resample(x.permute(0, 2, 1, 3, 4).reshape(b * t, x.shape[1], h, w))
        x = y.reshape(b, t, *y.shape[1:]).permute(0, 2, 1, 3, 4)
        if self.mode == "downsample3d" and cache is not None:
            slot = cache.take()
            prev = cache.slots[slot]
            if prev is None:                     # the first frame passes without a time step
                cache.slots[slot] = x.clone()
            else:
                keep = x[:, :, -1:].clone()
                x = self.time_conv(torch.cat((prev[:, :, -1:].to(x), x), 2))
                cache.slots[slot] = keep
        return x


def _run(layers, x, cache):
    for layer in layers:
        if isinstance(layer, (ResidualBlock, AttentionBlock, Resample)):
            x = layer(x, cache)
        elif isinstance(layer, CausalConv3d):
            x = _cached_conv(layer, x, cache)
        else:
            x = layer(x)
    return x


class Encoder3d(nn.Module):
    def __init__(self, dim=96, z_dim=32, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temporal_downsample=(False, True, True), dropout=0.0):
        super().__init__()
        dims = [dim * u for u in (1,) + tuple(dim_mult)]
        scale = 1.0
        self.conv1 = CausalConv3d(3, dims[0], 3, padding=1)
        blocks = []
        for i, (in_dim, out_dim) in enumerate(zip(dims[:-1], dims[1:])):
            for _ in range(num_res_blocks):
                blocks.append(ResidualBlock(in_dim, out_dim, dropout))
                if scale in attn_scales:
                    blocks.append(AttentionBlock(out_dim))
                in_dim = out_dim
            if i != len(dim_mult) - 1:
                blocks.append(Resample(out_dim, "downsample3d" if temporal_downsample[i] else "downsample2d"))
                scale /= 2.0
        self.downsamples = nn.Sequential(*blocks)
        self.middle = nn.Sequential(ResidualBlock(out_dim, out_dim, dropout), AttentionBlock(out_dim),
                                    ResidualBlock(out_dim, out_dim, dropout))
        self.head = nn.Sequential(ChannelRMSNorm(out_dim, images=False), nn.SiLU(),
                                  CausalConv3d(out_dim, z_dim, 3, padding=1))

    def forward(self, x, cache=None):
        x = _cached_conv(self.conv1, x, cache)
        x = _run(self.downsamples, x, cache)
        x = _run(self.middle, x, cache)
        return _run(self.head, x, cache)


class Decoder3d(nn.Module):
    def __init__(self, dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temporal_upsample=(True, True, False), dropout=0.0):
        super().__init__()
        dims = [dim * u for u in (dim_mult[-1],) + tuple(dim_mult[::-1])]
        scale = 1.0 / 2 ** (len(dim_mult) - 2)
        self.conv1 = CausalConv3d(z_dim, dims[0], 3, padding=1)
        self.middle = nn.Sequential(ResidualBlock(dims[0], dims[0], dropout), AttentionBlock(dims[0]),
                                    ResidualBlock(dims[0], dims[0], dropout))
        blocks = []
        for i, (in_dim, out_dim) in enumerate(zip(dims[:-1], dims[1:])):
            if i in (1, 2, 3):
                in_dim //= 2     # the previous stage's upsampling conv halved the width
            for _ in range(num_res_blocks + 1):
                blocks.append(ResidualBlock(in_dim, out_dim, dropout))
                if scale in attn_scales:
                    blocks.append(AttentionBlock(out_dim))
                in_dim = out_dim
            if i != len(dim_mult) - 1:
                blocks.append(Resample(out_dim, "upsample3d" if temporal_upsample[i] else "upsample2d"))
                scale *= 2.0
        self.upsamples = nn.Sequential(*blocks)
        self.head = nn.Sequential(ChannelRMSNorm(out_dim, images=False), nn.SiLU(),
                                  CausalConv3d(out_dim, 3, 3, padding=1))

    def forward(self, x, cache=None):
        x = _cached_conv(self.conv1, x, cache)
        x = _run(self.middle, x, cache)
        x = _run(self.upsamples, x, cache)
        return _run(self.head, x, cache)


class WanVAE(nn.Module):
    """``encode`` -> posterior mean (un-normalised latent), ``decode`` -> pixels in about [-1, 1]."""

    def __init__(self, dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temporal_downsample=(False, True, True), dropout=0.0):
        super().__init__()
        self.z_dim = z_dim
        self.encoder = Encoder3d(dim, 2 * z_dim, dim_mult, num_res_blocks, attn_scales, temporal_downsample, dropout)
        self.conv1 = CausalConv3d(2 * z_dim, 2 * z_dim, 1)
        self.conv2 = CausalConv3d(z_dim, z_dim, 1)
        self.decoder = Decoder3d(dim, z_dim, dim_mult, num_res_blocks, attn_scales, tuple(temporal_downsample[::-1]),
                                 dropout)

    def posterior(self, video):
        """``[B, 3, 1 + 4k, H, W]`` -> (mean, log-variance) ``[B, 16, 1 + k, H/8, W/8]``."""
        frames = video.shape[2]
        if (frames - 1) % 4:
            raise ValueError(f"Wan videos have 1 + 4k frames, got {frames}")
        cache, outs = _Cache(), []
        for start, stop in [(0, 1)] + [(1 + 4 * i, 5 + 4 * i) for i in range((frames - 1) // 4)]:
            cache.rewind()
            outs.append(self.encoder(video[:, :, start:stop], cache))
        mean, logvar = self.conv1(torch.cat(outs, 2)).chunk(2, dim=1)
        return mean, logvar

    def encode(self, video):
        return self.posterior(video)[0]

    def decode(self, latent):
        """``[B, 16, 1 + k, h, w]`` -> ``[B, 3, 1 + 4k, 8h, 8w]``."""
        x = self.conv2(latent)
        cache, outs = _Cache(), []
        for i in range(latent.shape[2]):
            cache.rewind()
            outs.append(self.decoder(x[:, :, i:i + 1], cache))
        return torch.cat(outs, 2)
