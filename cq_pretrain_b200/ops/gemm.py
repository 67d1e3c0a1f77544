"""GEMM entry points used by every linear layer.

On CUDA (bf16, dims multiples of 16) these run the hand-written sm_100a tcgen05/TMA kernel in
``csrc/gemm.cu``: TMA stages A/B tiles into 128B-swizzled shared memory, one elected thread
issues ``tcgen05.mma`` into a TMEM accumulator, and epilogue warps read TMEM with
``tcgen05.ld`` and apply bias / fp32 accumulate-into-``main_grad`` before storing. Other shapes
and CPU tensors use ``torch.matmul`` (the oracle).
"""

from __future__ import annotations

import os

import torch

from . import _ext

_MIN = 16


def _kernel_ok(*ts):
    if not _ext.cuda_kernels_enabled():
        return False
    for t in ts:
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.data_ptr() % 16 == 0):
            return False
    return True


def _aligned(m, n, k):
    return m >= 1 and n % 16 == 0 and k % 16 == 0 and n >= _MIN and k >= _MIN


def linear(x, weight, bias=None):
    """``x @ weight^T + bias`` with x ``[..., K]``, weight ``[N, K]``."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    n, k = weight.shape
    if _kernel_ok(x2, weight) and _ext.has("gemm_nt") and _aligned(x2.shape[0], n, k) and x2.shape[0] > 0:
        y = _ext.ops().gemm_nt(x2.contiguous(), weight.contiguous(), bias.to(torch.bfloat16) if bias is not None else None)
    else:
        y = torch.nn.functional.linear(x2, weight.to(x2.dtype), None if bias is None else bias.to(x2.dtype))
    return y.reshape(*shape[:-1], n)


def matmul_nn(a, b):
    """``a @ b`` with a ``[M, K]``, b ``[K, N]`` (the dX = dY W product)."""
    shape = a.shape
    a2 = a.reshape(-1, shape[-1])
    if _kernel_ok(a2, b) and _ext.has("gemm_nn") and _aligned(a2.shape[0], b.shape[1], b.shape[0]) and a2.shape[0] > 0:
        y = _ext.ops().gemm_nn(a2.contiguous(), b.contiguous())
    else:
        y = a2 @ b.to(a2.dtype)
    return y.reshape(*shape[:-1], b.shape[1])


def matmul_tn(a, b):
    """``a^T @ b`` with a ``[M, N]``, b ``[M, K]`` -> ``[N, K]`` (the weight-gradient product), fp32.

    On CUDA this is the tcgen05 TN kernel accumulating into a zeroed fp32 buffer (an fp32 copy of
    the operands would run on CUDA cores, an order of magnitude slower).
    """
    if a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
        out = torch.zeros(a.shape[1], b.shape[1], dtype=torch.float32, device=a.device)
        return matmul_tn_accumulate(a, b, out)
    return a.float().T @ b.float()


def matmul_tn_accumulate(a, b, out):
    """``out += a^T @ b`` accumulated in fp32 (``out`` fp32 ``[N, K]``)."""
    if _kernel_ok(a, b) and _ext.has("gemm_tn_acc") and out.is_cuda and out.dtype == torch.float32 \
            and a.shape[1] % 16 == 0 and b.shape[1] % 16 == 0 and a.shape[0] > 0 and out.is_contiguous():
        _ext.ops().gemm_tn_acc(a.contiguous(), b.contiguous(), out)
        return out
    if a.is_cuda:
        out.view(a.shape[1], b.shape[1]).addmm_(a.T, b, beta=1.0, alpha=1.0) if a.dtype == torch.float32 else \
            out.view(a.shape[1], b.shape[1]).add_(torch.mm(a.T, b, out_dtype=torch.float32) if _has_out_dtype() else (a.T @ b).float())
        return out
    out.view(a.shape[1], b.shape[1]).addmm_(a.float().T, b.float())
    return out


_OUT_DTYPE = None


def _has_out_dtype():
    global _OUT_DTYPE
    if _OUT_DTYPE is None:
        try:
            a = torch.zeros(16, 16, dtype=torch.bfloat16, device="cuda")
            torch.mm(a, a, out_dtype=torch.float32)
            _OUT_DTYPE = True
        except Exception:
            _OUT_DTYPE = False
    return _OUT_DTYPE
