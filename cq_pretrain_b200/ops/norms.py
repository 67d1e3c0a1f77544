"""Normalisation ops: Qwen RMSNorm (1+w), GDN gated RMSNorm, Wan adaLN modulate and gated residual.

CUDA bf16/fp32 tensors run the row kernels of ``csrc/rowops.cu`` (one warp per row, fp32
statistics, fused backward with an fp32 weight-gradient reduction); CPU runs ``reference``.
"""

from __future__ import annotations

import torch

from . import _ext
from . import reference as R


def _use_kernel(x):
    return x.is_cuda and _ext.has("rms_norm_fwd") and x.dtype in (torch.bfloat16, torch.float32)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = _ext.ops().rms_norm_fwd(x.contiguous(), weight.contiguous(), eps)
        ctx.save_for_backward(x, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        dx, dw = _ext.ops().rms_norm_bwd(dy.contiguous(), x.contiguous(), weight.contiguous(), rstd)
        return dx, dw.to(weight.dtype), None


def rms_norm(x, weight, eps):
    """Qwen RMSNorm ``x rsqrt(mean x^2 + eps) (1 + w)``."""
    if _use_kernel(x) and x.shape[-1] % 8 == 0:
        shape = x.shape
        return _RMSNorm.apply(x.reshape(-1, shape[-1]), weight, eps).reshape(shape)
    return R.rms_norm(x, weight, eps)


class _RMSNormResidual(torch.autograd.Function):
    """``(x, rms_norm(x))`` where ``x`` also feeds a residual connection: the backward receives the
    residual's gradient and the norm's, and one kernel returns their sum (no separate add)."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = _ext.ops().rms_norm_fwd(x.contiguous(), weight.contiguous(), eps)
        ctx.save_for_backward(x, weight, rstd)
        return x.view_as(x), y

    @staticmethod
    def backward(ctx, dres, dy):
        x, weight, rstd = ctx.saved_tensors
        if dy is None:
            return dres, None, None
        dx, dw = _ext.ops().rms_norm_bwd(dy.contiguous(), x.contiguous(), weight.contiguous(), rstd,
                                         None if dres is None else dres.contiguous())
        return dx, dw.to(weight.dtype), None


class _AddRMSNormResidual(torch.autograd.Function):
    """``(s, rms_norm(s))`` with ``s = x + branch`` computed in the norm's kernel; backward: one
    kernel gives ``ds`` (norm gradient plus the residual gradient of ``s``), which is the gradient
    of both ``x`` and ``branch``."""

    @staticmethod
    def forward(ctx, x, branch, weight, eps):
        y, rstd, s = _ext.ops().rms_norm_fwd(x.contiguous(), weight.contiguous(), eps, branch.contiguous())
        ctx.save_for_backward(s, weight, rstd)
        return s, y

    @staticmethod
    def backward(ctx, dres, dy):
        s, weight, rstd = ctx.saved_tensors
        if dy is None:
            return dres, dres, None, None
        ds, dw = _ext.ops().rms_norm_bwd(dy.contiguous(), s, weight.contiguous(), rstd,
                                         None if dres is None else dres.contiguous())
        return ds, ds, dw.to(weight.dtype), None


def add_rms_norm_residual(x, branch, weight, eps):
    """``(x + branch, rms_norm(x + branch))`` (the reference's ``add_rms_norm``) for 2-D tensors
    whose sum continues along the residual stream: one kernel each way."""
    if (_use_kernel(x) and x.dim() == 2 and x.shape[-1] % 8 == 0 and x.is_contiguous() and branch.shape == x.shape
            and branch.dtype == x.dtype):
        return _AddRMSNormResidual.apply(x, branch, weight, eps)
    return rms_norm_residual(x + branch, weight, eps)


def rms_norm_residual(x, weight, eps):
    """``(x, rms_norm(x))`` for a 2-D ``x`` that is also a residual input (see ``_RMSNormResidual``)."""
    if _use_kernel(x) and x.dim() == 2 and x.shape[-1] % 8 == 0 and x.is_contiguous():
        return _RMSNormResidual.apply(x, weight, eps)
    return x, rms_norm(x, weight, eps)


class _GatedNorm(torch.autograd.Function):
    """x ``[rows, D]``; z either the same shape or, at D = 128, ``[tokens, heads, 128]`` with any token
    stride (the gate slice of the GDN projection, read in place instead of copied)."""

    @staticmethod
    def forward(ctx, x, z, weight, eps):
        y, rstd = _ext.ops().gated_norm_fwd(x.contiguous(), z, weight.contiguous(), eps)
        ctx.save_for_backward(x, z, weight, rstd)
        ctx.z_shape = z.shape
        return y

    @staticmethod
    def backward(ctx, dy):
        x, z, weight, rstd = ctx.saved_tensors
        dx, dz, dw = _ext.ops().gated_norm_bwd(dy.contiguous(), x, z, weight, rstd)
        return dx, dz.view(ctx.z_shape), dw.to(weight.dtype), None


def gated_rms_norm(x, z, weight, eps):
    """``rms(x) * w * silu(z)`` over the last dim (one GDN head)."""
    if _use_kernel(x) and x.shape[-1] % 8 == 0 and z.dtype == x.dtype:
        shape = x.shape
        zk = z if (z.dim() == 3 and shape[-1] == 128 and z.stride(-1) == 1 and z.stride(-2) == 128) \
            else z.reshape(-1, shape[-1])
        return _GatedNorm.apply(x.reshape(-1, shape[-1]), zk, weight, eps).reshape(shape)
    return R.gated_rms_norm(x, z, weight, eps)


class _Modulate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, shift, index, eps):
        y, mean, rstd = _ext.ops().ln_modulate_fwd(x.contiguous(), scale.contiguous(), shift.contiguous(), index, eps)
        ctx.save_for_backward(x, scale, index, mean, rstd)
        ctx.nmod = scale.shape[0]
        return y

    @staticmethod
    def backward(ctx, dy):
        x, scale, index, mean, rstd = ctx.saved_tensors
        dx, dscale, dshift = _ext.ops().ln_modulate_bwd(dy.contiguous(), x, scale, index, mean, rstd)
        return dx, dscale, dshift, None, None


def layer_norm_modulate(x, scale, shift, eps, index=None):
    """``LN(x) (1 + scale[index]) + shift[index]`` in fp32; ``index`` maps rows to modulation rows."""
    if _use_kernel(x) and x.shape[-1] % 8 == 0 and scale.dtype == torch.float32:
        idx = index if index is not None else torch.arange(x.shape[0], device=x.device)
        return _Modulate.apply(x, scale, shift, idx.to(torch.int32).contiguous(), eps)
    if index is not None:
        scale, shift = scale.index_select(0, index), shift.index_select(0, index)
    return R.layer_norm_modulate(x, scale, shift, eps)


class _GatedAdd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, branch, gate, index):
        y = _ext.ops().gated_add_fwd(x.contiguous(), branch.contiguous(), gate.contiguous(), index)
        ctx.save_for_backward(branch, gate, index)
        return y

    @staticmethod
    def backward(ctx, dy):
        branch, gate, index = ctx.saved_tensors
        dbranch, dgate = _ext.ops().gated_add_bwd(dy.contiguous(), branch, gate, index)
        return dy, dbranch, dgate, None


def gated_add(x, branch, gate, index=None):
    """fp32 ``x + gate[index] * branch``."""
    if _use_kernel(x) and x.dtype == torch.float32 and gate.dtype == torch.float32 and x.shape[-1] % 8 == 0:
        idx = index if index is not None else torch.arange(x.shape[0], device=x.device)
        return _GatedAdd.apply(x, branch, gate, idx.to(torch.int32).contiguous())
    if index is not None:
        gate = gate.index_select(0, index)
    return R.gated_add(x, branch, gate)


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, wq, wk, cos, sin, head_dim, total_dim, eps, exchange):
        wqf, wkf = wq.float().contiguous(), wk.float().contiguous()
        yq, yk, rstd = _ext.ops().qk_norm_rope_fwd(q, k, wqf, wkf, cos=cos, sin=sin, head_dim=head_dim,
                                                   total_dim=total_dim, eps=eps, **(exchange() if exchange else {}))
        ctx.save_for_backward(q, k, wqf, wkf, rstd, cos, sin)
        ctx.meta = (head_dim, total_dim, exchange, wq.dtype)
        return yq, yk

    @staticmethod
    def backward(ctx, dyq, dyk):
        q, k, wqf, wkf, rstd, cos, sin = ctx.saved_tensors
        head_dim, total_dim, exchange, wdtype = ctx.meta
        zeros = lambda: torch.zeros(q.shape, dtype=torch.bfloat16, device=q.device)
        dyq = zeros() if dyq is None else dyq.to(torch.bfloat16)
        dyk = zeros() if dyk is None else dyk.to(torch.bfloat16)
        dq, dk, dwq, dwk = _ext.ops().qk_norm_rope_bwd(dyq, dyk, q, k, wqf, wkf, rstd, cos=cos, sin=sin,
                                                       head_dim=head_dim, total_dim=total_dim,
                                                       **(exchange() if exchange else {}))
        return dq, dk, dwq.to(wdtype), dwk.to(wdtype), None, None, None, None, None, None


def qk_norm_rope_supported(q, k):
    return (q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and q.dim() == 2
            and q.shape == k.shape and q.shape[1] % 8 == 0 and q.shape[1] <= 2048
            and all(t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 for t in (q, k))
            and _ext.has("qk_norm_rope_fwd"))


def qk_norm_rope(q, k, wq, wk, cos, sin, head_dim, total_dim, eps, exchange=None):
    """Wan self-attention q / k: ``rope(rms_norm(q) * wq)`` and the same for k in one kernel each way.

    ``q``, ``k`` ``[rows, D]`` bf16 (row-strided views allowed) hold this rank's heads of a
    ``total_dim``-wide vector; the norm's per-row sums run over the full width, so at TP > 1
    ``exchange()`` returns the peer-exchange arguments of one call (``SymmetricWorkspace.
    exchange_kwargs``) and the sums cross NVLink inside the kernel. ``cos`` / ``sin`` fp32 ``[rows,
    head_dim / 2]`` (the complex-pair RoPE angles) or None for the norm alone. Returns contiguous
    ``[rows, D]`` outputs. Reference: ``norm_q`` / ``norm_k`` and then ``rotary`` on q and k in
    ``models/generator_wan21.py:109-113``, three separate operations there."""
    if cos is not None:
        cos, sin = cos.float().contiguous(), sin.float().contiguous()
    return _QKNormRope.apply(q, k, wq, wk, cos, sin, head_dim, total_dim, eps, exchange)
