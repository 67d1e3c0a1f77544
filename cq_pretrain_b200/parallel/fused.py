"""Compute + collective pairs of the sequence-parallel linears.

* ``gather_linear``: all-gather the row shards, then ``X W^T`` (column-parallel forward).
* ``linear_scatter``: ``X W^T`` then reduce-scatter rows (row-parallel forward; also the
  column-parallel input gradient ``dY W``).

On CUDA with the symmetric-memory workspace (``parallel/symmetric.py``) these run as single
kernels that move tiles over NVLink peer memory while the tensor cores work (``csrc/comm.cu``):
the all-gather copies peer shards into the local gather buffer tile by tile and the GEMM
consumes them as they land; the GEMM->reduce-scatter stores each output tile into the owning
rank's buffer and reduces on arrival. NCCL + GEMM is the baseline path used everywhere else.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm
from . import state as ps


def gather_rows_raw(x):
    st = ps.state()
    if st.tp == 1:
        return x
    out = x.new_empty((x.shape[0] * st.tp, *x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def scatter_rows_raw(x):
    st = ps.state()
    if st.tp == 1:
        return x
    out = x.new_empty((x.shape[0] // st.tp, *x.shape[1:]))
    dist.reduce_scatter_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def _symm():
    from . import symmetric
    return symmetric.workspace()


def gather_linear(x, weight, bias=None):
    """Return ``(all_gather(x) @ W^T + b, all_gather(x))``."""
    ws = _symm()
    if ws is not None and ws.supports_gather(x, weight):
        return ws.gather_linear(x, weight, bias)
    xg = gather_rows_raw(x)
    return gemm.linear(xg, weight, bias), xg


def gather_matmul(dy, weight):
    """Return ``(all_gather(dY) @ W, all_gather(dY))`` (input gradient of a row-parallel linear)."""
    ws = _symm()
    if ws is not None and ws.supports_gather(dy, weight, transposed=True):
        return ws.gather_matmul(dy, weight)
    dyg = gather_rows_raw(dy)
    return gemm.matmul_nn(dyg, weight), dyg


def linear_scatter(x, weight, bias=None):
    """Return ``reduce_scatter(x @ W^T) + b`` (the bias is added once, by the rows' owner)."""
    ws = _symm()
    if ws is not None and ws.supports_scatter(x, weight):
        return ws.linear_scatter(x, weight, bias)
    y = scatter_rows_raw(gemm.linear(x, weight))
    return y if bias is None else y + bias.to(y.dtype)


def linear_scatter_grad(dy, weight, dy2=None, weight2=None):
    """Return ``reduce_scatter(dY @ W [+ pad(dY2) @ W2])``: the input gradient of one column-parallel
    linear, or of two that read the same gathered rows (``dY2`` covers the first ``len(dY2)`` rows)."""
    ws = _symm()
    if ws is not None and ws.supports_scatter(dy, weight, True, dy2, weight2):
        return ws.matmul_scatter(dy, weight, dy2, weight2)
    dx = gemm.matmul_nn(dy, weight)
    if dy2 is not None:
        dx[: dy2.shape[0]] += gemm.matmul_nn(dy2, weight2)
    return scatter_rows_raw(dx)
