"""Chunked, recomputed linear cross-entropy over a vocabulary-parallel weight.

For each chunk of rows: ``logits = h W_local^T`` (fp32), the row max, target logit and sum of
exponentials are combined across the TP group, and ``loss = log(sum) + max - target``. No
``[rows, vocab]`` tensor survives the forward; backward recomputes each chunk, forms
``dlogits = softmax - onehot``, and accumulates ``dW`` in fp32 (straight into ``main_grad`` when
present) and ``dh = dlogits W_local`` (summed over TP by the caller's row collective).
Reference: ``ops/cross_entropy.py:17-116``.

On CUDA the per-chunk work is an LM-head GEMM whose epilogue computes the row statistics
online (``csrc/gemm.cu``, epilogue 3), so logits are never written to memory in the forward,
and the backward recomputes each logits tile and stores ``(softmax - onehot) * dloss`` straight
from the accumulator (epilogue 4). Under TP the per-tile partials go straight into one kernel that
merges them, exchanges each row's (max, sum exp, target logit) with the other ranks over NVLink peer
memory and forms the full-vocabulary log-sum-exp (``csrc/comm.cu``, ``parallel/symmetric.py``); the
NCCL MAX + SUM all-reduce pair remains only for other devices or without the TP workspace.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _ext
from . import gemm
from ..parallel import state as ps


def _stats_combine(mx, tgt, sexp, group):
    """Merge per-rank (max, target logit, sum exp relative to the local max) into global values."""
    if group is None:
        return mx, tgt, sexp
    gmax = mx.clone()
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    packed = torch.stack((tgt, sexp * torch.exp(mx - gmax)))
    dist.all_reduce(packed, group=group)
    return gmax, packed[0], packed[1]


def _kernel_shapes(h, w):
    """The tcgen05 LM-head kernels need bf16 operands with K and the vocab shard multiples of 16."""
    return (h.is_cuda and _ext.cuda_kernels_enabled() and h.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and h.shape[1] % 16 == 0 and w.shape[0] % 16 == 0 and h.shape[0] > 0 and w.is_contiguous())


def _chunk_stats(h, w, targets, lo):
    """Local (max, target logit (0 if not owned), sum exp relative to local max) for one chunk."""
    if _kernel_shapes(h, w) and hasattr(_ext.ops(), "ce_stats"):
        return _ext.ops().ce_stats(h.contiguous(), w, targets, lo)
    logits = gemm.linear(h, w).float()
    mx = logits.max(-1).values
    local = targets - lo
    owned = (local >= 0) & (local < w.shape[0])
    tgt = logits.gather(1, local.clamp(0, w.shape[0] - 1)[:, None])[:, 0] * owned
    sexp = torch.exp(logits - mx[:, None]).sum(-1)
    return mx, tgt, sexp


def _fused_workspace(hidden, weight, group, chunk):
    """The TP workspace when the in-kernel statistics exchange applies (CUDA kernels, TP > 1)."""
    if group is None or not _kernel_shapes(hidden, weight) or not _ext.has("ce_partials"):
        return None
    from ..parallel import symmetric
    ws = symmetric.workspace()
    return ws if ws is not None and ws.supports_ce(min(chunk, hidden.shape[0])) else None


DLOGITS_BUDGET = 4 << 30   # bytes of bf16 softmax gradients the kernel path may hold at once


def _rows_per_pass(chunk, rows, vocab_shard, kernel):
    """Rows per LM-head pass. ``chunk`` bounds memory on small devices; on the kernel path the
    passes grow to a 4 GiB bf16 gradient buffer, because every pass's weight-gradient GEMM reads
    and writes the whole fp32 ``main_grad`` of the head (2 GB at 248K x 2048)."""
    if not kernel:
        return chunk
    fit = max(chunk, (DLOGITS_BUDGET // max(1, vocab_shard * 2)) // 128 * 128)
    return max(1, min(rows, fit))


class _LinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, chunk, group, rank):
        chunk = _rows_per_pass(chunk, hidden.shape[0], weight.shape[0], _kernel_shapes(hidden, weight))
        lo = rank * weight.shape[0]
        total = torch.zeros((), dtype=torch.float32, device=hidden.device)
        lse_all = torch.empty(hidden.shape[0], dtype=torch.float32, device=hidden.device)
        ws = _fused_workspace(hidden, weight, group, chunk)
        for start in range(0, hidden.shape[0], chunk):
            h, t = hidden[start:start + chunk], targets[start:start + chunk]
            if ws is not None:
                lse, tgt = ws.ce_combine(*_ext.ops().ce_partials(h.contiguous(), weight, t, lo))
            else:
                mx, tgt, sexp = _stats_combine(*_chunk_stats(h, weight, t, lo), group)
                lse = mx + torch.log(sexp)
            lse_all[start:start + chunk] = lse
            total += (lse - tgt).sum()
        ctx.save_for_backward(hidden, weight, targets, lse_all)
        ctx.chunk, ctx.lo = chunk, lo
        return total / max(1, hidden.shape[0])

    @staticmethod
    def backward(ctx, grad_out):
        hidden, weight, targets, lse_all = ctx.saved_tensors
        factor = grad_out.float() / max(1, hidden.shape[0])
        dh = torch.empty_like(hidden)
        mg = getattr(weight, "main_grad", None)
        dw = mg if mg is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        n = weight.shape[0]
        for start in range(0, hidden.shape[0], ctx.chunk):
            h, t = hidden[start:start + ctx.chunk], targets[start:start + ctx.chunk]
            lse = lse_all[start:start + ctx.chunk]
            if _kernel_shapes(h, weight) and hasattr(_ext.ops(), "ce_grad_logits"):
                grad = _ext.ops().ce_grad_logits(h.contiguous(), weight, t, lse, ctx.lo, factor)
            else:
                logits = gemm.linear(h, weight).float()
                prob = torch.exp(logits - lse[:, None])
                local = t - ctx.lo
                owned = (local >= 0) & (local < n)
                prob.scatter_add_(1, local.clamp(0, n - 1)[:, None], -owned[:, None].to(prob.dtype))
                grad = (prob * factor).to(hidden.dtype)
            dh[start:start + ctx.chunk] = gemm.matmul_nn(grad, weight).to(dh.dtype)
            gemm.matmul_tn_accumulate(grad, h, dw)
        if mg is not None:
            cb = getattr(weight, "_grad_ready", None)
            if cb is not None:
                cb(weight)
            return dh, None, None, None, None, None
        return dh, dw.to(weight.dtype), None, None, None, None


def linear_cross_entropy(hidden, weight, targets, chunk):
    """Mean CE of ``hidden @ W_full^T`` against ``targets``; ``weight`` is this rank's vocab shard.

    ``hidden`` must be identical on every TP rank; its gradient is the local-vocab part, which
    the caller's row collective sums across ranks.
    """
    st = ps.state()
    group = st.tp_group if st.tp > 1 else None
    return _LinearCE.apply(hidden, weight, targets, chunk, group, st.tp_rank)
