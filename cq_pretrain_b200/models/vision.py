"""Qwen3.5-style vision tower + 2x2 merger producing backbone-width visual content tokens.

Patch projection (Conv3d 2x16x16 weights run as a GEMM), bilinear learned absolute position
embedding, pre-LN blocks with 2-D rotary varlen attention (each image / frame block attends
within itself) and GELU-tanh MLPs, then a merger (LN, concat of 2x2 neighbours, MLP) to the
backbone width (reference ``models/vision_encoder.py:13-235``). By default the encoder and merger
are frozen (no grad, eval), and the trainer can consume cached merger features instead.

Vision TP (``vision_tensor_parallel``, reference ``models/vision_encoder.py:45-54``): with TP > 1
the qkv (fused, sharded per head with stride 3), fc1 and merger fc1 weights are column shards and
proj, fc2 and merger fc2 row shards, Megatron style on replicated activations: a column layer's
input gradient is summed over TP, a row layer's output is summed over TP (then its replicated
bias added). Each rank runs attention on its own heads.
"""

from __future__ import annotations

from contextlib import nullcontext

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import attention as ATT
from ..ops import reference as R
from ..parallel import layers as P
from ..parallel import state as ps

DEFAULT = dict(depth=12, hidden_size=768, intermediate_size=3072, num_heads=12, num_position_embeddings=2304,
               out_hidden_size=1024, patch_size=16, spatial_merge_size=2, temporal_patch_size=2, in_channels=3)


def vision_config(cfg):
    """Tower geometry for a run config (tiny configs get a tiny tower)."""
    tp = bool(getattr(cfg, "vision_tensor_parallel", False))
    if cfg.width >= 1024:
        return dict(DEFAULT, depth=24, hidden_size=1024, intermediate_size=4096, num_heads=16,
                    out_hidden_size=cfg.width, tensor_parallel=tp)
    return dict(DEFAULT, depth=2, hidden_size=64, intermediate_size=128, num_heads=4, num_position_embeddings=256,
                out_hidden_size=cfg.width, tensor_parallel=tp)


def _tp(cfg):
    return bool(cfg.get("tensor_parallel")) and ps.tp_size() > 1


def column(cfg, in_features, out_features, stride=1):
    return P.column_linear(in_features, out_features, stride=stride, parallel=_tp(cfg))


def row(cfg, in_features, out_features):
    return P.row_linear(in_features, out_features, parallel=_tp(cfg))


apply_column, apply_row = P.apply_column, P.apply_row


class VisionBlock(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        d = cfg["hidden_size"]
        tp = ps.tp_size() if _tp(cfg) else 1
        if cfg["num_heads"] % tp:
            raise ValueError(f"vision heads {cfg['num_heads']} not divisible by TP={tp}")
        self.heads = cfg["num_heads"] // tp
        self.head_dim = d // cfg["num_heads"]
        self.norm1 = nn.LayerNorm(d, eps=1e-6)
        self.norm2 = nn.LayerNorm(d, eps=1e-6)
        self.qkv = column(cfg, d, 3 * d, stride=3)
        self.proj = row(cfg, d, d)
        self.fc1 = column(cfg, d, cfg["intermediate_size"])
        self.fc2 = row(cfg, cfg["intermediate_size"], d)

    def forward(self, x, layout):
        n = x.shape[0]
        hd = self.head_dim
        q, k, v = apply_column(self.qkv, self.norm1(x)).reshape(n, 3, self.heads, hd).unbind(1)
        q = R.rotary_half(q, layout.cos, layout.sin, hd)
        k = R.rotary_half(k, layout.cos, layout.sin, hd)
        y = ATT.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), layout.ends, layout.ends)
        x = x + apply_row(self.proj, y.reshape(n, self.heads * hd))
        return x + apply_row(self.fc2, F.gelu(apply_column(self.fc1, self.norm2(x)), approximate="tanh"))


class VisionTower(nn.Module):
    def __init__(self, cfg=None, out_width=None, freeze_encoder=True, freeze_merger=True):
        super().__init__()
        cfg = dict(DEFAULT, **(cfg or {}))
        self.cfg = cfg
        d = cfg["hidden_size"]
        m = cfg["spatial_merge_size"]
        patch_in = cfg["in_channels"] * cfg["temporal_patch_size"] * cfg["patch_size"] ** 2
        self.patch_embed = nn.Linear(patch_in, d)
        self.pos_embed = nn.Embedding(cfg["num_position_embeddings"], d)
        self.blocks = nn.ModuleList([VisionBlock(cfg) for _ in range(cfg["depth"])])
        self.merge_width = d * m * m
        self.merger_norm = nn.LayerNorm(d, eps=1e-6)
        self.merger_fc1 = column(cfg, self.merge_width, self.merge_width)
        self.merger_fc2 = row(cfg, self.merge_width, cfg["out_hidden_size"])
        out_width = out_width or cfg["out_hidden_size"]
        self.bridge = nn.Identity() if out_width == cfg["out_hidden_size"] else nn.Linear(cfg["out_hidden_size"], out_width, bias=False)
        if _tp(cfg):
            P.mark_duplicates(self)   # replicated activations: full gradients on every TP rank
        self.freeze_encoder, self.freeze_merger = freeze_encoder, freeze_merger
        if freeze_encoder:
            for mod in (self.patch_embed, self.pos_embed, self.blocks):
                mod.requires_grad_(False)
        if freeze_merger:
            for mod in (self.merger_norm, self.merger_fc1, self.merger_fc2, self.bridge):
                mod.requires_grad_(False)

    def head_dim(self):
        return self.cfg["hidden_size"] // self.cfg["num_heads"]

    def encode(self, layout):
        x = self.patch_embed(layout.pixel_values.to(self.patch_embed.weight.dtype))
        pos = self.pos_embed(layout.pos_indices) * layout.pos_weights.to(x.dtype)[..., None]
        x = x + pos.sum(0)
        for block in self.blocks:
            x = block(x, layout)
        return x

    def forward(self, layout):
        with torch.no_grad() if self.freeze_encoder else nullcontext():
            x = self.encode(layout)
        with torch.no_grad() if self.freeze_merger else nullcontext():
            merged = self.merger_norm(x).reshape(-1, self.merge_width)
            out = apply_row(self.merger_fc2, F.gelu(apply_column(self.merger_fc1, merged)))
            return self.bridge(out)
