"""Linear layers whose weight gradient accumulates straight into an FP32 ``main_grad``.

``y = x W^T + b``. Backward computes ``dX = dY W`` and ``main_grad += dY^T X`` in FP32 without
materialising a bf16 ``dW`` (reference ``ops/functional.py:31-36`` + ``distributed/megatron.py:45-49``,
the ``gradient_accumulation_fusion`` contract). When a parameter has no ``main_grad`` (no
optimizer wrapper) the gradient is returned normally. After accumulating, the parameter's
``_grad_ready`` callback (set by the data-parallel wrapper) marks it ready so bucket
reduce-scatters can start while backward continues.

CUDA tensors run the sm_100a GEMM (``gemm.cu``); the fused TP variants run the
all-gather->GEMM / GEMM->reduce-scatter kernels of ``parallel/fused.py`` when available.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _ext
from . import gemm


def _accumulate(param, grad):
    """Add ``grad`` (fp32 or bf16) into ``param.main_grad`` and fire readiness; returns the autograd grad."""
    if param is None:
        return None
    mg = getattr(param, "main_grad", None)
    if mg is None:
        return grad.to(param.dtype)
    mg.add_(grad.view_as(mg))
    cb = getattr(param, "_grad_ready", None)
    if cb is not None:
        cb(param)
    return None


def _bias_grad(dy):
    """Column sums of ``dy`` in fp32 (one kernel reading bf16 directly on CUDA)."""
    dy2 = dy.reshape(-1, dy.shape[-1])
    if dy2.is_cuda and _ext.cuda_kernels_enabled() and _ext.has("column_sum") and dy2.shape[1] % 8 == 0:
        return _ext.ops().column_sum(dy2)
    return dy2.float().sum(0)


def _weight_grad(param, dy, x):
    """``main_grad += dy^T x`` (fp32 accumulate) or return ``dy^T x``."""
    mg = getattr(param, "main_grad", None)
    if mg is not None:
        gemm.matmul_tn_accumulate(dy, x, mg)
        cb = getattr(param, "_grad_ready", None)
        if cb is not None:
            cb(param)
        return None
    return gemm.matmul_tn(dy, x).to(param.dtype)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        ctx.bias = bias
        return gemm.linear(x, weight, bias)

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm.matmul_nn(dy, weight) if ctx.needs_input_grad[0] else None
        dw = _weight_grad(weight, dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])) if ctx.needs_input_grad[1] else None
        db = _accumulate(ctx.bias, _bias_grad(dy)) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def linear(x, weight, bias=None):
    if not (x.requires_grad or weight.requires_grad or (bias is not None and bias.requires_grad)):
        return gemm.linear(x, weight, bias)
    return _Linear.apply(x, weight, bias)


class _GatherLinear(torch.autograd.Function):
    """Column-parallel: ``y = all_gather_rows(x) @ W^T (+ b)``; backward reduce-scatters dX."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        from ..parallel import fused
        y, xg = fused.gather_linear(x, weight, bias)
        ctx.save_for_backward(xg, weight)
        ctx.has_bias, ctx.bias = bias is not None, bias
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..parallel import fused
        xg, weight = ctx.saved_tensors
        dy = dy.contiguous()
        dx = fused.linear_scatter_grad(dy, weight) if ctx.needs_input_grad[0] else None
        dw = _weight_grad(weight, dy, xg) if ctx.needs_input_grad[1] else None
        db = _accumulate(ctx.bias, _bias_grad(dy)) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def gather_linear(x, weight, bias=None):
    return _GatherLinear.apply(x, weight, bias)


class _GatherLinearPair(torch.autograd.Function):
    """Two column-parallel projections of one all-gathered input: ``y1 = xg W1^T + b1`` (the
    all-gather runs inside this GEMM) and ``y2 = xg[:rows2] W2^T + b2`` on the gathered rows.
    Backward: ``reduce_scatter(dY1 W1 + pad(dY2) W2)`` in one GEMM -> reduce-scatter kernel."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, rows2):
        from ..parallel import fused
        y1, xg = fused.gather_linear(x, w1, b1)
        x2 = xg if rows2 is None else xg[:rows2]
        y2 = gemm.linear(x2, w2, b2)
        ctx.save_for_backward(xg, w1, w2)
        ctx.rows2, ctx.b1, ctx.b2 = rows2, b1, b2
        return y1, y2

    @staticmethod
    def backward(ctx, dy1, dy2):
        from ..parallel import fused
        xg, w1, w2 = ctx.saved_tensors
        rows2 = xg.shape[0] if ctx.rows2 is None else ctx.rows2
        dy1 = torch.zeros(xg.shape[0], w1.shape[0], dtype=xg.dtype, device=xg.device) if dy1 is None else dy1.contiguous()
        dy2 = torch.zeros(rows2, w2.shape[0], dtype=xg.dtype, device=xg.device) if dy2 is None else dy2.contiguous()
        dx = fused.linear_scatter_grad(dy1, w1, dy2, w2) if ctx.needs_input_grad[0] else None
        dw1 = _weight_grad(w1, dy1, xg) if ctx.needs_input_grad[1] else None
        dw2 = _weight_grad(w2, dy2, xg[:rows2]) if ctx.needs_input_grad[3] else None
        db1 = _accumulate(ctx.b1, _bias_grad(dy1)) if ctx.b1 is not None and ctx.needs_input_grad[2] else None
        db2 = _accumulate(ctx.b2, _bias_grad(dy2)) if ctx.b2 is not None and ctx.needs_input_grad[4] else None
        return dx, dw1, db1, dw2, db2, None


def gather_linear_pair(x, w1, b1, w2, b2, rows2=None):
    """``(all_gather(x) W1^T + b1, all_gather(x)[:rows2] W2^T + b2)`` with one all-gather."""
    return _GatherLinearPair.apply(x, w1, b1, w2, b2, rows2)


class _LinearScatter(torch.autograd.Function):
    """Row-parallel: ``y = reduce_scatter_rows(x @ W^T) + b``; backward all-gathers dY inside the
    input-gradient GEMM (``all_gather(dY) @ W``) and reuses the gathered rows for the weight gradient."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        from ..parallel import fused
        ctx.save_for_backward(x, weight)
        ctx.has_bias, ctx.bias = bias is not None, bias
        return fused.linear_scatter(x, weight, bias)

    @staticmethod
    def backward(ctx, dy):
        from ..parallel import fused
        x, weight = ctx.saved_tensors
        if ctx.needs_input_grad[0]:
            dx, dyg = fused.gather_matmul(dy.contiguous(), weight)   # one all-gather->GEMM kernel
        else:
            dx, dyg = None, fused.gather_rows_raw(dy.contiguous())
        dw = _weight_grad(weight, dyg, x) if ctx.needs_input_grad[1] else None
        db = _accumulate(ctx.bias, _bias_grad(dy)) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def linear_scatter(x, weight, bias=None):
    return _LinearScatter.apply(x, weight, bias)
