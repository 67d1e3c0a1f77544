"""Attention ops.

``cq_attention``: softmax attention of CQ rows over content keys where row ``r`` sees the key
range ``[kstart[r], kend[r])`` (the planner's exact visibility); GQA; rows with an empty range
output zero. ``varlen_attention``: non-causal packed attention inside each sample (Wan self
and cross attention; ``q_ends``/``k_ends`` cumulative).

CUDA runs the tcgen05 flash-attention kernels of ``csrc/attention.cu``: TMA-fed tiles, scores
and accumulators in tensor memory, the mask computed on the fly from the two range vectors with
exact key-tile skipping, fp32 softmax; the backward recomputes P from the saved LSE in a dQ
kernel over row blocks and a dK/dV kernel over key blocks (deterministic, no atomics). CPU runs
``reference`` (SDPA with the mask built per row tile).
"""

from __future__ import annotations

import torch

from . import _ext
from . import reference as R


def _kernel(q):
    return q.is_cuda and _ext.cuda_kernels_enabled() and q.dtype == torch.bfloat16 and q.shape[-1] in (64, 128, 256) \
        and hasattr(_ext.ops(), "attn_fwd")


class _RangeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, kstart, kend, scale):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = _ext.ops().attn_fwd(q, k, v, kstart, kend, scale)
        ctx.save_for_backward(q, k, v, o, lse, kstart, kend)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, kstart, kend = ctx.saved_tensors
        dq, dk, dv = _ext.ops().attn_bwd(do.contiguous(), q, k, v, o, lse, kstart, kend, ctx.scale)
        return dq, dk, dv, None, None, None


def cq_attention(q, k, v, kstart, kend, scale=None):
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    if _kernel(q):
        return _RangeAttention.apply(q, k, v, kstart.to(torch.int32).contiguous(), kend.to(torch.int32).contiguous(), scale)
    return R.range_attention(q, k, v, kstart, kend, scale)


def ranges_from_ends(q_ends, k_ends, device):
    """Per-query-row key ranges for packed samples (row of sample i sees keys of sample i)."""
    qs, ks, ke = [], [], []
    qa = ka = 0
    for qb, kb in zip(q_ends, k_ends):
        qs.append((qb - qa, ka, kb))
        qa, ka = qb, kb
    n = sum(x[0] for x in qs)
    kstart = torch.empty(n, dtype=torch.int32)
    kend = torch.empty(n, dtype=torch.int32)
    r = 0
    for count, a, b in qs:
        kstart[r:r + count] = a
        kend[r:r + count] = b
        r += count
    return kstart.to(device, non_blocking=True), kend.to(device, non_blocking=True)


def varlen_attention(q, k, v, q_ends, k_ends, scale=None, ranges=None):
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    if _kernel(q):
        kstart, kend = ranges if ranges is not None else ranges_from_ends(q_ends, k_ends, q.device)
        return _RangeAttention.apply(q, k, v, kstart, kend, scale)
    return R.varlen_attention(q, k, v, q_ends, k_ends, scale)
