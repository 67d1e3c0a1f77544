"""Legacy flow renderer and RGB patch embedding, kept for regression tests of old checkpoints.

``FlowRenderer`` is a small DiT that denoises a square grid of latent tokens (``image_tokens``
positions of ``latent_channels`` each) conditioned on the backbone's query outputs through
cross-attention (reference ``models/legacy.py:11-130``):

* conditions ``[n, Q, width]`` -> ``memory_proj(condition_proj(.))`` (computed once and shared by
  the ``flow_draws`` noise draws);
* ``xt = (1 - t) noise + t x0`` per draw; the time embedding is a 256-wide sinusoid of ``1000 t``
  through a SiLU MLP;
* blocks: adaLN (6 modulations from the time) -> self-attention with 2-D rotary positions (the
  first half of each head dim rotates with the row, the second with the column) -> LayerNorm ->
  cross-attention to the memory -> adaLN -> GELU-tanh MLP, gated residuals;
* zero-initialised modulation and output layers, so an untrained renderer predicts 0;
* loss = mean over draws, tokens and channels of ``(v_hat - (x0 - noise))^2``.

``RGBPatchLinear`` embeds raw RGB images as 16x16 patches with a GEMM in the Conv2d weight
layout (``[width, 3, p, p]``). Both run replicated (TP = 1).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import attention as ATT
from ..ops import reference as R


class RGBPatchLinear(nn.Module):
    def __init__(self, width, patch_size):
        super().__init__()
        self.patch_size = patch_size
        self.weight = nn.Parameter(torch.empty(width, 3, patch_size, patch_size))
        self.bias = nn.Parameter(torch.empty(width))
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        bound = 1 / math.sqrt(3 * patch_size ** 2)
        nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, pixels):
        """pixels ``[n, 3, H, W]`` -> tokens ``[n, (H/p)(W/p), width]`` in row-major patch order."""
        n, c, h, w = pixels.shape
        p = self.patch_size
        x = pixels.reshape(n, c, h // p, p, w // p, p).permute(0, 2, 4, 1, 3, 5).reshape(n, -1, c * p * p)
        return F.linear(x, self.weight.flatten(1).to(x.dtype), self.bias.to(x.dtype))


def _modulate(x, scale, shift):
    return F.layer_norm(x.float(), (x.shape[-1],), eps=1e-6).to(x.dtype) * (1 + scale) + shift


class _Attention(nn.Module):
    def __init__(self, cfg, cross):
        super().__init__()
        self.heads, self.dim, self.cross = cfg.dit_heads, cfg.dit_width // cfg.dit_heads, cross
        d = cfg.dit_width
        if cross:
            self.q, self.kv = nn.Linear(d, d), nn.Linear(d, 2 * d)
        else:
            self.qkv = nn.Linear(d, 3 * d)
        self.out = nn.Linear(d, d)

    def forward(self, x, rope=None, memory=None):
        """x ``[B, T, D]``; memory ``[B, M, D]``; attention runs per sample as packed varlen."""
        b, t, d = x.shape
        if self.cross:
            q = self.q(x).reshape(b * t, self.heads, self.dim)
            m = memory.shape[1]
            k, v = self.kv(memory).reshape(b * m, 2, self.heads, self.dim).unbind(1)
            k_ends = tuple(range(m, b * m + 1, m))
        else:
            q, k, v = self.qkv(x).reshape(b * t, 3, self.heads, self.dim).unbind(1)
            cos, sin = rope
            half = self.dim // 2
            q = torch.cat((R.rotary_half(q[..., :half], cos[0], sin[0], half),
                           R.rotary_half(q[..., half:], cos[1], sin[1], half)), -1)
            k = torch.cat((R.rotary_half(k[..., :half], cos[0], sin[0], half),
                           R.rotary_half(k[..., half:], cos[1], sin[1], half)), -1)
            k_ends = tuple(range(t, b * t + 1, t))
        q_ends = tuple(range(t, b * t + 1, t))
        y = ATT.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), q_ends, k_ends)
        return self.out(y.reshape(b, t, d))


class _Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        d = cfg.dit_width
        self.self_attn, self.cross_attn = _Attention(cfg, False), _Attention(cfg, True)
        self.ada = nn.Linear(d, 6 * d)
        self.up, self.down = nn.Linear(d, cfg.dit_ffn), nn.Linear(cfg.dit_ffn, d)
        nn.init.zeros_(self.ada.weight)
        nn.init.zeros_(self.ada.bias)

    def forward(self, x, time, memory, rope):
        shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = self.ada(F.silu(time)).chunk(6, -1)
        x = x + gate_a * self.self_attn(_modulate(x, scale_a, shift_a), rope=rope)
        x = x + self.cross_attn(F.layer_norm(x, (x.shape[-1],), eps=1e-6), memory=memory)
        return x + gate_m * self.down(F.gelu(self.up(_modulate(x, scale_m, shift_m)), approximate="tanh"))


class FlowRenderer(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        d = cfg.dit_width
        self.condition_proj = nn.Linear(cfg.width, cfg.width)
        self.memory_proj = nn.Linear(cfg.width, d)
        self.input_proj = nn.Linear(cfg.latent_channels, d)
        self.time_embed = nn.Sequential(nn.Linear(256, d), nn.SiLU(), nn.Linear(d, d))
        self.blocks = nn.ModuleList([_Block(cfg) for _ in range(cfg.dit_layers)])
        self.final_ada = nn.Linear(d, 2 * d)
        self.output = nn.Linear(d, cfg.latent_channels)
        for layer in (self.final_ada, self.output):
            nn.init.zeros_(layer.weight)
            nn.init.zeros_(layer.bias)
        self.register_buffer("freqs", torch.exp(-math.log(10000.0) * torch.arange(128).float() / 128),
                             persistent=False)
        side = math.isqrt(cfg.image_tokens)
        idx = torch.arange(cfg.image_tokens)
        half = cfg.dit_head_dim // 2
        inv = 10000.0 ** (-torch.arange(0, half, 2, dtype=torch.float64) / half)
        tables = []
        for pos in (idx // side, idx % side):          # row, column
            ang = pos[:, None].double() * inv
            ang = torch.cat((ang, ang), -1)
            tables.append((ang.cos().float(), ang.sin().float()))
        self.register_buffer("rope_cos", torch.stack([c for c, _ in tables]), persistent=False)
        self.register_buffer("rope_sin", torch.stack([s for _, s in tables]), persistent=False)

    def forward(self, conditions, batch):
        cfg = self.cfg
        draws = cfg.flow_draws
        x0 = batch.latents.float().repeat(draws, 1, 1)               # [F n, T, C]
        noise, t = batch.noise.float(), batch.times.float()
        xt = (1 - t[:, None, None]) * noise + t[:, None, None] * x0
        dtype = conditions.dtype
        memory = self.memory_proj(self.condition_proj(conditions)).repeat(draws, 1, 1)
        x = self.input_proj(xt.to(dtype))
        ang = t[:, None] * 1000 * self.freqs[None]
        time = self.time_embed(torch.cat((ang.cos(), ang.sin()), -1).to(dtype))[:, None]
        b, tokens = x.shape[:2]
        cos = self.rope_cos.to(dtype).repeat(1, b, 1)               # [2, B*T, half]
        sin = self.rope_sin.to(dtype).repeat(1, b, 1)
        for block in self.blocks:
            if cfg.checkpoint_dit and self.training and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(block, x, time, memory, (cos, sin), use_reentrant=False)
            else:
                x = block(x, time, memory, (cos, sin))
        shift, scale = self.final_ada(F.silu(time)).chunk(2, -1)
        v = self.output(_modulate(x, scale, shift)).float()
        return (v - (x0 - noise)).square().mean()
