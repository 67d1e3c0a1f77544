"""Row gathers whose backward is also a gather (no atomics, deterministic).

``rows(src, index, inverse)`` returns ``src[index]``. ``inverse`` is a tuple of int64 tensors,
one per multiplicity level: ``inverse[l][j]`` is the ``l``-th output row that reads source row
``j``, or ``len(index)`` (an appended zero row) when there is none. The plan precomputes these
on the host, so the backward is ``sum_l grad[inverse[l]]`` instead of an atomic index_add.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _ext


def inverse_levels(index, n_src, ignore=None):
    """Host-side inverse of a gather index (``ignore``: a source id whose gradient is discarded)."""
    index = np.asarray(index, dtype=np.int64)
    n = len(index)
    levels = []
    order = np.argsort(index, kind="stable")
    sorted_src = index[order]
    first = np.searchsorted(sorted_src, np.arange(n_src), side="left")
    last = np.searchsorted(sorted_src, np.arange(n_src), side="right")
    if ignore is not None and 0 <= ignore < n_src:
        last[ignore] = first[ignore]   # its readers get no gradient, so it sets no level
    depth = int((last - first).max()) if n_src else 0
    for level in range(depth):
        inv = np.full(n_src, n, dtype=np.int64)
        has = (last - first) > level
        inv[has] = order[first[has] + level]
        if ignore is not None and 0 <= ignore < n_src:
            inv[ignore] = n
        levels.append(inv)
    return tuple(torch.from_numpy(x) for x in levels)


class _Rows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, src, index, *inverse):
        ctx.inverse = inverse
        ctx.n_src = src.shape[0]
        return src.index_select(0, index)

    @staticmethod
    def backward(ctx, grad):
        padded = torch.cat((grad, grad.new_zeros(1, *grad.shape[1:])))
        out = None
        for inv in ctx.inverse:
            part = padded.index_select(0, inv)
            out = part if out is None else out + part
        if out is None:
            out = grad.new_zeros(ctx.n_src, *grad.shape[1:])
        return (out, None) + (None,) * len(ctx.inverse)


_STACKED: dict = {}


def _stacked(inverse):
    """The inverse levels as one ``[levels, n_src]`` device tensor (cached per plan tensor)."""
    key = (id(inverse[0]), len(inverse))
    hit = _STACKED.get(key)
    if hit is None or hit[0] is not inverse[0]:
        if len(_STACKED) > 256:
            _STACKED.clear()
        hit = (inverse[0], torch.stack(inverse).contiguous())
        _STACKED[key] = hit
    return hit[1]


class _RowsCuda(torch.autograd.Function):
    @staticmethod
    def forward(ctx, index, inv, src, second):
        ctx.inv, ctx.n0 = inv, src.shape[0]
        ctx.n1 = 0 if second is None else second.shape[0]
        return _ext.ops().gather_rows(src, second, index)

    @staticmethod
    def backward(ctx, grad):
        grads = _ext.ops().gather_rows_bwd(grad.contiguous(), ctx.inv, ctx.n0, ctx.n1)
        return None, None, grads[0], (grads[1] if ctx.n1 else None)


def _rows_aligned(t):
    """Rows contiguous inside, 16-byte aligned base and row stride (column slices qualify)."""
    if t.shape[0] == 0 or not t[0].is_contiguous():
        return False
    es = t.element_size()
    return t.data_ptr() % 16 == 0 and (t.shape[0] == 1 or (t.stride(0) * es) % 16 == 0)


def _cuda_ok(src, second, inverse):
    if not (src.is_cuda and _ext.cuda_kernels_enabled() and _ext.has("gather_rows")):
        return False
    if src.dtype not in (torch.bfloat16, torch.float32) or not _rows_aligned(src):
        return False
    if second is not None and (second.dtype != src.dtype or second.shape[1:] != src.shape[1:]
                               or not _rows_aligned(second)):
        return False
    width = src[0].numel()
    return (width * src.element_size()) % 16 == 0 and (inverse is None or width % 8 == 0)


def rows(src, index, inverse=None, second=None):
    """``cat(src, second)[index]`` where an index past the last source row reads zeros.

    ``inverse`` (levels over the concatenated sources, optionally plus one sentinel row) makes
    the backward a gather too. On CUDA one kernel gathers and one kernel sums the inverse levels
    (``csrc/gather.cu``); no zero row or concatenation is materialised.
    """
    needs_grad = src.requires_grad or (second is not None and second.requires_grad)
    if _cuda_ok(src, second, inverse if needs_grad else None):
        if inverse is None or not needs_grad:
            return _ext.ops().gather_rows(src, second, index)
        return _RowsCuda.apply(index, _stacked(inverse), src, second)
    parts = [src] + ([second] if second is not None else []) + [src.new_zeros(1, *src.shape[1:])]
    full = torch.cat(parts, 0)
    if inverse is None or not needs_grad:
        return full.index_select(0, index)
    n_src = inverse[0].numel() if inverse else full.shape[0]
    if n_src < full.shape[0]:
        full = full[:n_src]
    out = _Rows.apply(full, index, *inverse)
    return out
