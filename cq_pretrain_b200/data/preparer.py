"""Per-consumption flow randomness and host->device preparation of packed batches.

Flow noise, flow times and time features come from a private CPU generator seeded by
``sha256(snapshot, seed, epoch, rank, serial)`` (reference ``data/codec.py:69-71,128-134``), so
the draw depends only on which pack is consumed, never on prefetch depth or model RNG.
"""

from __future__ import annotations

import hashlib

import torch

from .batch import EmbeddingPlan, backbone_ids
from .generation import time_features


def consumption_seed(signature, serial) -> int:
    key = f"{signature['snapshot']}:{signature['seed']}:{signature['epoch']}:{signature['rank']}:{serial}"
    return int.from_bytes(hashlib.sha256(key.encode()).digest()[:8], "little") & ((1 << 63) - 1)


class FakeLatentEncoder:
    """Deterministic stand-in VAE for pipeline tests: average-pool + fixed channel projection."""

    def __init__(self, channels=16, stride=8):
        weight = torch.arange(channels * 3, dtype=torch.float32).reshape(-1, 3, 1, 1)
        self.projection = (weight.remainder(11) - 5) / 15
        self.stride = stride

    def encode(self, pixels):
        from torch.nn import functional as F
        x = F.avg_pool2d(pixels.float(), self.stride)
        return F.conv2d(x, self.projection.to(x.device))


class DevicePreparer:
    """Attach flow noise/times/time features to a host batch and return a device copy."""

    def __init__(self, cfg, device="cpu", dtype=torch.float32):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype

    def randomness(self, batch, receipt):
        layout = batch.generation
        legacy = self.cfg.renderer == "legacy" and batch.latents is not None
        if layout is None and not legacy:
            return None
        signature = receipt["next_state"]["documents"].get("signature") or dict(snapshot="synthetic", seed=0, epoch=0, rank=0)
        gen = torch.Generator().manual_seed(consumption_seed(signature, receipt["serial"]))
        if legacy:   # flow_draws noise draws per target, times ~ logit-normal
            n, tokens, channels = batch.latents.shape
            draws = self.cfg.flow_draws
            noise = torch.randn(draws * n, tokens, channels, generator=gen)
            times = torch.randn(draws * n, generator=gen).sigmoid().clamp(1e-5, 1 - 1e-5)
            return noise, times, None
        channels = self.cfg.latent_channels if self.cfg.renderer == "moss" else self.cfg.latent_channels * 4
        noise = torch.randn(sum(layout.lengths), channels, generator=gen)
        times = torch.randn(len(layout.lengths), generator=gen).sigmoid().clamp(1e-5, 1 - 1e-5)
        freq_dim = 256 if self.cfg.renderer == "moss" else self.cfg.wan_freq_dim   # MOSS: fixed 256-wide sinusoid
        return noise, times, time_features(times, freq_dim)

    def __call__(self, batch, receipt, non_blocking=False):
        """The device copy of ``batch`` with its flow randomness and the host-built sort plan of
        the backbone input ids (``EmbeddingPlan``); on CUDA the new host tensors are pinned so every
        copy is asynchronous."""
        extra = self.randomness(batch, receipt)
        pin = self.device.type == "cuda"
        if extra is not None:
            noise, times, feats = (t.pin_memory() if pin and t is not None else t for t in extra)
            batch.noise, batch.times = noise, times
            if batch.generation is not None:
                batch.generation.time_features = feats
            if batch.latents is None:
                raise ValueError("generation targets need latents (cached or encoded)")
        if batch.mainline is not None and batch.embed_plan is None and batch.ids.device.type == "cpu":
            plan = EmbeddingPlan.build(backbone_ids(batch, self.cfg.text_mask_token_id, self.cfg.image_mask_token_id))
            batch.embed_plan = plan.pin_memory() if pin else plan
        out = batch.to(self.device, non_blocking=non_blocking)
        if out.vision is not None and out.vision.features is not None:
            out.vision.features = out.vision.features.to(self.dtype)
        return out
