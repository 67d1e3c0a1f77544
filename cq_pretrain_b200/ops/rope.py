"""Rotary embeddings: Qwen partial rotate-half MRoPE and Wan complex-pair 3D RoPE."""

from __future__ import annotations

import torch

from . import _ext
from . import reference as R


def rotary_half(x, cos, sin, dim):
    return R.rotary_half(x, cos, sin, dim)


class _RopePairs(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin):
        ctx.save_for_backward(cos, sin)
        return _ext.ops().rope_pairs(x, cos, sin, False)

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        return _ext.ops().rope_pairs(dy.contiguous(), cos, sin, True), None, None


def rotary_pairs(x, cos, sin):
    """Wan complex-pair RoPE; one elementwise kernel each way on CUDA (the backward rotates back)."""
    if (x.is_cuda and x.dim() == 3 and x.shape[-1] % 8 == 0 and x.dtype in (torch.bfloat16, torch.float32)
            and _ext.has("rope_pairs")):
        return _RopePairs.apply(x.contiguous(), cos, sin)
    return R.rotary_pairs(x, cos, sin)
