"""Sequence-parallel tensor-parallel layers.

Between modules every activation is row-sharded across the TP group (``[rows/tp, width]``).
A column-parallel linear all-gathers the rows and multiplies by its output-column shard; a
row-parallel linear multiplies by its input-row shard and reduce-scatters the rows. This is
mathematically the reference's Megatron TP (column: identity fwd / all-reduce dX bwd; row:
all-reduce fwd, ``distributed/megatron.py:118-196``) with the all-reduce split into
reduce-scatter + all-gather around the row-local work (norms, residuals), which then runs on
1/tp of the rows. On CUDA the gather and scatter are fused into the GEMM kernels
(``parallel/fused.py``); NCCL is the baseline path.

Parameters carry ``tensor_model_parallel``, ``partition_dim``, ``partition_stride`` and optional
``_checkpoint_splits`` (logical fused-projection widths), as in the reference, so checkpoint
slicing and TP resharding can reconstruct official tensors.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import nn

from . import state as ps
from ..ops import _ext
from ..ops import linear as L


def mark_sharded(parameter, dim=0, stride=1, splits=None):
    parameter.tensor_model_parallel = True
    parameter.partition_dim = dim
    parameter.partition_stride = stride
    if splits is not None:
        parameter._checkpoint_splits = tuple(splits)
    return parameter


def normal_init(tensor, std=0.02, generator=None):
    return nn.init.normal_(tensor, std=std, generator=generator)


# ---- row (sequence) collectives -----------------------------------------------------------
def _gather_rows(x, group, world):
    out = x.new_empty((x.shape[0] * world, *x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _scatter_rows(x, group, world):
    out = x.new_empty((x.shape[0] // world, *x.shape[1:]))
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


class GatherRows(torch.autograd.Function):
    """All-gather row shards (forward) / reduce-scatter row gradients (backward)."""

    @staticmethod
    def forward(ctx, x):
        st = ps.state()
        return _gather_rows(x, st.tp_group, st.tp)

    @staticmethod
    def backward(ctx, grad):
        st = ps.state()
        return _scatter_rows(grad, st.tp_group, st.tp)


class ScatterRows(torch.autograd.Function):
    """Reduce-scatter partial rows (forward) / all-gather gradients (backward)."""

    @staticmethod
    def forward(ctx, x):
        st = ps.state()
        return _scatter_rows(x, st.tp_group, st.tp)

    @staticmethod
    def backward(ctx, grad):
        st = ps.state()
        return _gather_rows(grad, st.tp_group, st.tp)


class SplitRows(torch.autograd.Function):
    """Keep this rank's row shard of a replicated tensor (forward) / all-gather (backward)."""

    @staticmethod
    def forward(ctx, x):
        st = ps.state()
        n = x.shape[0] // st.tp
        return x[st.tp_rank * n:(st.tp_rank + 1) * n].contiguous()

    @staticmethod
    def backward(ctx, grad):
        st = ps.state()
        return _gather_rows(grad, st.tp_group, st.tp)


class ReduceTP(torch.autograd.Function):
    """Sum over the TP group (forward) / identity (backward): partial sums whose result every rank
    then uses identically (a loss, a replicated activation), so each rank's gradient of the sum is
    already the full one."""

    @staticmethod
    def forward(ctx, x):
        x = x.clone()
        dist.all_reduce(x, group=ps.state().tp_group)
        return x

    @staticmethod
    def backward(ctx, grad):
        return grad


class SumTP(torch.autograd.Function):
    """Sum over the TP group whose result each rank consumes differently (forward and backward
    both sum): e.g. per-row partial statistics that every rank applies to its own columns, so the
    gradient of the sum is the sum of every rank's contribution."""

    @staticmethod
    def forward(ctx, x):
        x = x.clone()
        dist.all_reduce(x, group=ps.state().tp_group)
        return x

    @staticmethod
    def backward(ctx, grad):
        grad = grad.clone()
        dist.all_reduce(grad, group=ps.state().tp_group)
        return grad


def sum_tp(x):
    return SumTP.apply(x) if ps.tp_size() > 1 else x


class CopyToTP(torch.autograd.Function):
    """Identity forward / sum over the TP group backward: a replicated input feeding
    column-sharded weights (each rank's input gradient is a partial sum)."""

    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        grad = grad.clone()
        dist.all_reduce(grad, group=ps.state().tp_group)
        return grad


def copy_to_tp(x):
    return CopyToTP.apply(x) if ps.tp_size() > 1 else x


class ReplicatedUse(torch.autograd.Function):
    """Identity forward; gradient divided by TP size.

    Marks a branch that every TP rank evaluates identically on a gathered tensor, so the
    gather's reduce-scatter backward (a sum over ranks) restores the exact gradient.
    """

    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        return grad / ps.tp_size()


def replicated_use(x):
    return ReplicatedUse.apply(x) if ps.tp_size() > 1 else x


def gather_rows(x):
    return GatherRows.apply(x) if ps.tp_size() > 1 else x


def scatter_rows(x):
    return ScatterRows.apply(x) if ps.tp_size() > 1 else x


def split_rows(x):
    return SplitRows.apply(x) if ps.tp_size() > 1 else x


def reduce_tp(x):
    return ReduceTP.apply(x) if ps.tp_size() > 1 else x


def local_row_range(rows: int):
    tp, r = ps.tp_size(), ps.tp_rank()
    n = rows // tp
    return r * n, (r + 1) * n


# ---- layers -------------------------------------------------------------------------------
class ColumnLinear(nn.Module):
    """``y[:, shard] = gather(x) @ W[shard]^T``; ``out_features`` split over TP (``stride`` for fused pairs)."""

    def __init__(self, in_features, out_features, bias=False, stride=1, splits=None):
        super().__init__()
        tp = ps.tp_size()
        if out_features % tp:
            raise ValueError(f"output width {out_features} not divisible by TP={tp}")
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features // tp, in_features))
        normal_init(self.weight)
        mark_sharded(self.weight, 0, stride, splits)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features // tp))
            mark_sharded(self.bias, 0, stride, splits)
        else:
            self.register_parameter("bias", None)

    def forward(self, x, gathered=False):
        if ps.tp_size() > 1 and not gathered:
            return L.gather_linear(x, self.weight, self.bias)
        return L.linear(x, self.weight, self.bias)


def column_pair(x, first, second, rows2=None):
    """Two column-parallel projections of the same row-sharded input: ``(first(gather(x)),
    second(gather(x)[:rows2]))``. Under TP the rows are gathered once, inside the first GEMM, and
    the backward sums both input gradients in one GEMM -> reduce-scatter kernel."""
    if ps.tp_size() > 1:
        return L.gather_linear_pair(x, first.weight, first.bias, second.weight, second.bias, rows2)
    return first(x), second(x if rows2 is None else x[:rows2])


class RowLinear(nn.Module):
    """``y = scatter(x[:, shard] @ W[:, shard]^T) + b``; ``in_features`` split over TP."""

    def __init__(self, in_features, out_features, bias=False):
        super().__init__()
        tp = ps.tp_size()
        if in_features % tp:
            raise ValueError(f"input width {in_features} not divisible by TP={tp}")
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features // tp))
        normal_init(self.weight)
        mark_sharded(self.weight, 1)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)

    def forward(self, x):
        if ps.tp_size() > 1:
            return L.linear_scatter(x, self.weight, self.bias)
        return L.linear(x, self.weight, self.bias)


# ---- Megatron-style TP on replicated activations (vision tower, MOSS renderer) --------------
def column_linear(in_features, out_features, bias=True, stride=1, parallel=True):
    """Output-sharded weights under TP (``parallel`` and TP > 1), else a plain ``nn.Linear``."""
    if parallel and ps.tp_size() > 1:
        return ColumnLinear(in_features, out_features, bias=bias, stride=stride)
    return nn.Linear(in_features, out_features, bias=bias)


def row_linear(in_features, out_features, bias=True, parallel=True):
    if parallel and ps.tp_size() > 1:
        return RowLinear(in_features, out_features, bias=bias)
    return nn.Linear(in_features, out_features, bias=bias)


def apply_column(layer, x):
    """Column shard on a replicated input: ``x W_shard^T + b_shard`` (input grad summed over TP)."""
    if isinstance(layer, ColumnLinear):
        return L.linear(copy_to_tp(x), layer.weight, layer.bias)
    return layer(x)


def apply_row(layer, x):
    """Row shard: ``sum_TP(x_shard W_shard^T) + b`` (replicated output)."""
    if isinstance(layer, RowLinear):
        y = reduce_tp(L.linear(x, layer.weight))
        return y if layer.bias is None else y + layer.bias.to(y.dtype)
    return layer(x)


def mark_duplicates(module):
    """Replicated-activation TP: every rank computes the full gradient of the module's
    unsharded parameters, so the optimizer must not sum them over TP."""
    if ps.tp_size() > 1:
        for p in module.parameters():
            if not getattr(p, "tensor_model_parallel", False):
                p.tp_duplicate = True
    return module


class VocabEmbedding(nn.Module):
    """Vocabulary-parallel embedding; output is row-sharded (partial lookups reduce-scattered)."""

    def __init__(self, vocab, width):
        super().__init__()
        tp = ps.tp_size()
        if vocab % tp:
            raise ValueError("vocabulary must divide TP")
        self.vocab, self.width = vocab, width
        self.weight = nn.Parameter(torch.empty(vocab // tp, width))
        normal_init(self.weight)
        mark_sharded(self.weight, 0)

    def partial(self, ids, plan=None):
        """This rank's masked lookup ``[n, width]`` (full rows, zero outside the local vocab range).

        On CUDA the lookup is the row-gather kernel (ids outside this shard hit the zero sentinel)
        and the backward adds each token id's rows straight into the FP32 ``main_grad`` rows it
        touches (``rows_accumulate``: a deterministic sum per id), instead of building a dense
        vocabulary gradient and adding it. ``plan`` (``data.batch.EmbeddingPlan`` of ``ids``, built
        on the host) gives the backward its sort order; without it the backward sorts on the device
        and reads the run lengths back to the host."""
        n = self.weight.shape[0]
        lo = ps.tp_rank() * n
        local = ids - lo
        owned = (local >= 0) & (local < n)
        if (ids.is_cuda and self.weight.dtype == torch.bfloat16 and self.weight.shape[1] % 8 == 0
                and _ext.has("rows_accumulate")):
            sort = None
            if plan is not None and plan.order.numel() == ids.numel():
                runs = plan.run_ids - lo
                runs = torch.where((runs >= 0) & (runs < n), runs, torch.full_like(runs, n))   # other shards: skipped
                sort = (plan.order, plan.seg_start, plan.run_seg, runs)
            return _EmbeddingLookup.apply(torch.where(owned, local, torch.full_like(local, n)), self.weight, sort)
        out = nn.functional.embedding(local.clamp(0, n - 1), self.weight)
        if ps.tp_size() > 1:
            out = out * owned[:, None].to(out.dtype)
        return out

    def forward(self, ids):
        return scatter_rows(self.partial(ids))


def _segments(counts, seg=16):
    """Cut runs of ``counts`` sorted positions into segments of at most ``seg`` positions:
    ``(segment boundaries [segments + 1], first segment of every run [runs + 1])`` (int64, host)."""
    pieces = (counts + seg - 1) // seg
    run_seg = torch.zeros(len(counts) + 1, dtype=torch.long)
    torch.cumsum(pieces, 0, out=run_seg[1:])
    run_start = torch.zeros(len(counts), dtype=torch.long)
    run_start[1:] = torch.cumsum(counts, 0)[:-1]
    owner = torch.repeat_interleave(torch.arange(len(counts)), pieces)
    within = torch.arange(int(run_seg[-1])) - run_seg[:-1][owner]
    starts = run_start[owner] + within * seg
    return torch.cat((starts, counts.sum().reshape(1))), run_seg


class _EmbeddingLookup(torch.autograd.Function):
    """``weight[index]`` with ``index == len(weight)`` reading a zero row."""

    @staticmethod
    def forward(ctx, index, weight, sort):
        ctx.save_for_backward(index)
        ctx.weight, ctx.sort = weight, sort
        return _ext.ops().gather_rows(weight, None, index.contiguous())

    @staticmethod
    def backward(ctx, grad):
        (index,) = ctx.saved_tensors
        weight = ctx.weight
        if ctx.sort is not None:
            order, seg_start, run_seg, ids = ctx.sort
        else:
            order = torch.argsort(index, stable=True)
            ids, counts = torch.unique_consecutive(index.index_select(0, order), return_counts=True)
            seg_start, run_seg = _segments(counts.cpu())
            seg_start = seg_start.to(index.device, non_blocking=True)
            run_seg = run_seg.to(index.device, non_blocking=True)
        # runs of other shards' ids (== len(weight)) are skipped by the kernel
        mg = getattr(weight, "main_grad", None)
        target = mg if mg is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        _ext.ops().rows_accumulate(grad.contiguous(), order, seg_start, run_seg, ids.contiguous(), target)
        if mg is not None:
            cb = getattr(weight, "_grad_ready", None)
            if cb is not None:
                cb(weight)
            return None, None, None
        return None, target.to(weight.dtype), None


def checkpoint_shard(value, parameter):
    """Slice a full (official) tensor into this rank's TP view, honouring stride and logical splits."""
    if ps.tp_size() == 1 or not getattr(parameter, "tensor_model_parallel", False):
        return value
    dim, rank, size = parameter.partition_dim, ps.tp_rank(), ps.tp_size()
    splits = getattr(parameter, "_checkpoint_splits", None)
    if splits is not None:
        return torch.cat([part.chunk(size, dim=dim)[rank] for part in value.split(splits, dim=dim)], dim=dim)
    stride = getattr(parameter, "partition_stride", 1)
    chunks = value.split(value.shape[dim] // size // stride, dim=dim)
    return torch.cat(chunks[rank::size], dim=dim)
