"""Rotary embeddings: Qwen partial rotate-half MRoPE and Wan complex-pair 3D RoPE."""

from __future__ import annotations

from . import reference as R


def rotary_half(x, cos, sin, dim):
    return R.rotary_half(x, cos, sin, dim)


def rotary_pairs(x, cos, sin):
    return R.rotary_pairs(x, cos, sin)
