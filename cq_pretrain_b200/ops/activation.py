"""Activations. SwiGLU (``silu(gate) * up`` over the two halves) runs as a bf16 row kernel on CUDA."""

from __future__ import annotations

import torch

from . import _ext
from . import reference as R


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return _ext.ops().swiglu_fwd(x.contiguous())

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return _ext.ops().swiglu_bwd(dy.contiguous(), x)


def swiglu(x):
    if x.is_cuda and _ext.has("swiglu_fwd") and x.dtype == torch.bfloat16 and x.shape[-1] % 16 == 0:
        shape = x.shape
        return _SwiGLU.apply(x.reshape(-1, shape[-1])).reshape(*shape[:-1], shape[-1] // 2)
    return R.swiglu(x)


def gelu_tanh(x):
    return torch.nn.functional.gelu(x, approximate="tanh")
