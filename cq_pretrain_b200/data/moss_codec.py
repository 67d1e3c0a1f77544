"""MOSS latent codec: the frozen FLUX.2 VAE posterior, 2x2 packing and the VAE's learned
batch-norm statistics (reference ``data/moss_codec.py:1-87``).

* ``pack``: ``[B, C, H, W]`` -> ``[B, 4C, H/2, W/2]`` with channel order (c, dy, dx), so one latent
  token covers 16 x 16 pixels (the FLUX.2 VAE downsamples by 8);
* ``normalize_posterior``: packed posterior mean / std standardised by the VAE's BN running
  statistics, ``(mean - mu) / sqrt(var + eps)`` and ``std / sqrt(var + eps)``;
* ``FrozenMOSSEncoder``: loads the pinned MOSS-Image-Base VAE through ``diffusers``
  (``AutoencoderKLFlux2``, optional; the error names it when missing), keeps only the encoder on
  the device, and encodes uint8-range pixels scaled to [-1, 1] in chunks;
* ``draw_latents``: one posterior draw ``mean + std * eps`` per latent token, tokens row-major.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

MOSS_VAE_REVISION = "1ceede80badddd6a7812069619edaa5633587192"


def pack(x: torch.Tensor) -> torch.Tensor:
    b, c, h, w = x.shape
    if h % 2 or w % 2:
        raise ValueError("packing needs even latent height and width")
    return x.reshape(b, c, h // 2, 2, w // 2, 2).permute(0, 1, 3, 5, 2, 4).reshape(b, c * 4, h // 2, w // 2)


def normalize_posterior(mean, std, running_mean, running_var, eps):
    """Packed posterior statistics standardised by the BN running statistics (fp32)."""
    mu = running_mean.float().view(1, -1, 1, 1)
    inv = torch.rsqrt(running_var.float() + eps).view(1, -1, 1, 1)
    return (pack(mean.float()) - mu) * inv, pack(std.float()) * inv


def draw_latents(means, stds, generator=None):
    """Per-target ``[C, h, w]`` statistics -> ``[sum h*w, C]`` token latents of one posterior draw."""
    tokens = [m.flatten(1).T for m in means]
    scales = [s.flatten(1).T for s in stds]
    mean, std = torch.cat(tokens), torch.cat(scales)
    noise = torch.randn(mean.shape, generator=generator, dtype=mean.dtype).to(mean.device)
    return mean + std * noise


class FrozenMOSSEncoder:
    def __init__(self, assets, device="cpu", dtype=torch.float32, chunk=1):
        root = Path(assets)
        manifest = json.loads((root / "manifest.json").read_text())
        if manifest.get("revision") != MOSS_VAE_REVISION:
            raise ValueError("unexpected MOSS VAE revision")
        try:
            from diffusers import AutoencoderKLFlux2
        except ImportError as error:
            raise ImportError("encoding MOSS latents needs diffusers (AutoencoderKLFlux2)") from error
        self.vae = AutoencoderKLFlux2.from_pretrained(str(root / "vae"), local_files_only=True, torch_dtype=dtype)
        self.vae.requires_grad_(False).eval()
        self.vae.encoder.to(device)
        self.vae.quant_conv.to(device)
        self.dtype, self.chunk, self.device = dtype, chunk, device

    @torch.no_grad()
    def encode(self, pixels):
        """uint8-range ``[B, 3, H, W]`` -> (standardised packed means, stds) ``[B, 4C, H/16, W/16]``."""
        bn = self.vae.bn
        means, stds = [], []
        for i in range(0, len(pixels), self.chunk):
            x = pixels[i:i + self.chunk].to(self.device, self.dtype) / 127.5 - 1
            posterior = self.vae.encode(x).latent_dist
            m, s = normalize_posterior(posterior.mean, posterior.std, bn.running_mean, bn.running_var,
                                       self.vae.config.batch_norm_eps)
            means.append(m)
            stds.append(s)
        return torch.cat(means), torch.cat(stds)
