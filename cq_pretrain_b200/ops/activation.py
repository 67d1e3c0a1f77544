"""Activations. SwiGLU (``silu(gate) * up`` over the two halves) runs as a bf16 row kernel on CUDA;
the MOSS renderer's SITU, affine modulation and gated residual run as fp32-math kernels of
``csrc/moss.cu`` (strided row slices read in place)."""

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


# ---- MOSS renderer pointwise ops (csrc/moss.cu) ----------------------------------------------
SITU, AFFINE, GATED_ADD = 0, 1, 2


def situ_reference(hidden, gate):
    """SITU of MOSS-Image-Base: ``(4 tanh(g/4) sigmoid(g)) * (25 tanh(h/25))`` in fp32."""
    h, g = hidden.float(), gate.float()
    return ((4 * torch.tanh(g / 4) * torch.sigmoid(g)) * (25 * torch.tanh(h / 25))).to(hidden.dtype)


def affine_reference(hidden, scale, shift):
    return (hidden.float() * (1 + scale.float()) + shift.float()).to(hidden.dtype)


def gated_add_reference(hidden, branch, gate):
    return (hidden.float() + branch.float() * gate.float()).to(hidden.dtype)


class _MossPointwise(torch.autograd.Function):
    @staticmethod
    def forward(ctx, kind, a, b, c):
        ctx.kind = kind
        ctx.save_for_backward(a, b, c)
        return _ext.ops().moss_pointwise_fwd(kind, a, b, c)

    @staticmethod
    def backward(ctx, dy):
        a, b, c = ctx.saved_tensors
        d0, d1 = _ext.ops().moss_pointwise_bwd(ctx.kind, dy.contiguous(), a, b, c)
        if ctx.kind == SITU:
            return None, d0, d1, None
        if ctx.kind == AFFINE:
            return None, d0, d1, dy
        return None, dy, d0, d1


def _moss_kernel(*xs):
    x = xs[0]
    return (x.is_cuda and x.dim() == 2 and x.dtype in (torch.bfloat16, torch.float32) and x.shape[1] % 8 == 0
            and _ext.has("moss_pointwise_fwd")
            and all(t.shape == x.shape and t.dtype == x.dtype and t.stride(1) == 1
                    and (t.shape[0] <= 1 or t.stride(0) * t.element_size() % 16 == 0)
                    and t.data_ptr() % 16 == 0 for t in xs))


def situ(hidden, gate):
    if _moss_kernel(hidden, gate):
        return _MossPointwise.apply(SITU, hidden, gate, hidden)
    return situ_reference(hidden, gate)


def affine(hidden, scale, shift):
    if _moss_kernel(hidden, scale, shift):
        return _MossPointwise.apply(AFFINE, hidden, scale, shift)
    return affine_reference(hidden, scale, shift)


def gated_add(hidden, branch, gate):
    if _moss_kernel(hidden, branch, gate):
        return _MossPointwise.apply(GATED_ADD, hidden, branch, gate)
    return gated_add_reference(hidden, branch, gate)
