"""Frozen Wan2.1 VAE codec: RGB video <-> normalised latents (reference ``data/wan_codec.py:8-65``).

The normalisation is part of the latent-cache contract: ``encode`` returns the posterior mean of
``models.wan_vae.WanVAE`` standardised per channel, ``(z - mean_c) / std_c``, and ``decode``
inverts it before the decoder. The per-channel statistics are the published ones of the Wan2.1
VAE (``LATENT_MEAN`` / ``LATENT_STD``); a ``config.json`` next to the checkpoint with
``latents_mean`` / ``latents_std`` overrides them.

* ``encode(rgb)``: ``[3, 1 + 4k, H, W]`` in [-1, 1], H and W multiples of 16 ->
  ``[16, 1 + k, H/8, W/8]`` fp32 (posterior mean, not a sample, as the native pipeline does).
* ``encode_images(x)``: ``[B, 3, H, W]`` -> ``[B, 16, H/8, W/8]`` (one-frame videos), the interface
  the latent cache preparer calls.
* ``decode(latents)``: a list of ``[16, 1 + k, h, w]`` -> list of ``[3, 1 + 4k, 8h, 8w]`` clamped to
  [-1, 1].
* ``from_pretrained(path)``: the published ``Wan2.1_VAE.pth`` (or a directory holding it) loaded
  strictly into ``WanVAE``.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..models.wan_vae import WanVAE

LATENT_MEAN = (-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508,
               0.4134, -0.0715, 0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921)
LATENT_STD = (2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743,
              3.2687, 2.1526, 2.8652, 1.5579, 1.6382, 1.1253, 2.8251, 1.9160)


class WanVideoCodec:
    def __init__(self, vae: WanVAE, mean=LATENT_MEAN, std=LATENT_STD):
        self.vae = vae.eval().requires_grad_(False)
        if len(mean) != vae.z_dim or len(std) != vae.z_dim:
            raise ValueError("latent statistics must have one value per latent channel")
        self.mean = torch.tensor(mean, dtype=torch.float32).view(-1, 1, 1, 1)
        self.std = torch.tensor(std, dtype=torch.float32).view(-1, 1, 1, 1)

    @classmethod
    def from_pretrained(cls, path, device="cpu", dtype=torch.float32):
        path = Path(path)
        folder = path if path.is_dir() else path.parent
        if path.is_dir():
            path = path / "Wan2.1_VAE.pth"
        state = torch.load(path, map_location="cpu", weights_only=True)
        state = state.get("state_dict", state)
        vae = WanVAE(dim=int(state["encoder.conv1.weight"].shape[0]))   # 96 for the published VAE
        vae.load_state_dict(state, strict=True)
        mean, std = LATENT_MEAN, LATENT_STD
        config = folder / "config.json"
        if config.is_file():
            meta = json.loads(config.read_text())
            mean, std = tuple(meta.get("latents_mean", mean)), tuple(meta.get("latents_std", std))
        return cls(vae.to(device=device, dtype=dtype), mean, std)

    def _param(self):
        return next(self.vae.parameters())

    @torch.no_grad()
    def encode(self, rgb):
        if rgb.dim() != 4 or rgb.shape[0] != 3 or (rgb.shape[1] - 1) % 4 or rgb.shape[2] % 16 or rgb.shape[3] % 16:
            raise ValueError(f"Wan RGB must be [3, 1 + 4k, H, W] with H, W multiples of 16, got {tuple(rgb.shape)}")
        p = self._param()
        with torch.autocast(p.device.type, enabled=False):
            z = self.vae.encode(rgb[None].to(p)).float()[0]
        return (z - self.mean.to(z)) / self.std.to(z)

    @torch.no_grad()
    def encode_images(self, images):
        return torch.stack([self.encode(x[:, None])[:, 0] for x in images])

    @torch.no_grad()
    def decode(self, latents):
        p = self._param()
        out = []
        for z in latents:
            raw = z.float() * self.std.to(z.device) + self.mean.to(z.device)
            with torch.autocast(p.device.type, enabled=False):
                out.append(self.vae.decode(raw[None].to(p)).float()[0].clamp(-1, 1))
        return out

    def frames(self, latent):
        """``decode`` of one latent ``[16, 1 + k, h, w]`` as ``[1 + 4k, 8h, 8w, 3]`` in [0, 1]: the
        ``decode`` callback of ``eval.sampling.generate`` (its visuals go to PNG / MP4)."""
        video = self.decode([latent])[0]
        return ((video + 1) / 2).permute(1, 2, 3, 0).cpu()
