"""Row gathers whose backward is also a gather (no atomics, deterministic).

``rows(src, index, inverse)`` returns ``src[index]``. ``inverse`` is a tuple of int64 tensors,
one per multiplicity level: ``inverse[l][j]`` is the ``l``-th output row that reads source row
``j``, or ``len(index)`` (an appended zero row) when there is none. The plan precomputes these
on the host, so the backward is ``sum_l grad[inverse[l]]`` instead of an atomic index_add.
"""

from __future__ import annotations

import numpy as np
import torch


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


def rows(src, index, inverse=None):
    if inverse is None or not src.requires_grad:
        return src.index_select(0, index)
    return _Rows.apply(src, index, *inverse)
