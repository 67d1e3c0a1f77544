"""Gated DeltaNet ops: chunked gated delta rule over CQ event streams and the causal short conv.

``gated_delta`` takes event-ordered q, k ``[E, H, Dk]``, v ``[E, H, Dv]``, log-decay g and
beta ``[E, H]`` (fp32) and per-document event boundaries; q/k are L2-normalised inside
(``use_qk_l2norm_in_kernel``). Read-only query events carry k = v = 0, beta = 0, g = 0, so they
read the state without changing it (reference ``ops/gated_delta_net.py:143-214``).

CUDA runs ``csrc/gdn.cu``: a chunk-parallel kernel builds the WY factors (T = (I+A)^-1, W, U)
for every 64-event chunk, a per-(document, head) kernel carries the 128x128 fp32 state across
chunks, and the backward mirrors both passes in reverse. CPU runs the chunked reference.
"""

from __future__ import annotations

import torch

from . import _ext
from . import reference as R


def _kernel(q):
    return q.is_cuda and _ext.cuda_kernels_enabled() and hasattr(_ext.ops(), "gdn_fwd")


def gated_delta(q, k, v, g, beta, bounds, chunk=64):
    if _kernel(q):
        from .gdn_cuda import gated_delta_cuda
        return gated_delta_cuda(q, k, v, g, beta, bounds, chunk)
    return R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk).to(v.dtype)


def prefill(q, k, v, g, beta, bounds, chunk=64):
    """Inference prefill: ``(outputs [E, H, Dv], final state per document [docs, H, Dk, Dv] fp32)``;
    on CUDA the forward recurrence kernel writes the final states (reference
    ``ops/gated_delta_net.py:293-312``)."""
    if _kernel(q):
        from .gdn_cuda import gated_delta_cuda
        return gated_delta_cuda(q, k, v, g, beta, bounds, chunk, final=True)
    y, state = R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk, final=True)
    return y.to(v.dtype), state


class _ConvAndQuery(torch.autograd.Function):
    """``updates = raw[content_order]``, ``conv = causal_conv_silu(updates)`` and
    ``query = query_conv_silu(raw, updates)`` as one node. Backward, with no zero-fill or add of a
    full gradient: the conv backward writes d_updates, the query history gradient is added into it in
    place, the inverse gather writes every row of d_raw (zero where no content row came from), and
    the queries' own-projection gradient then overwrites their (zero) rows of d_raw; content and
    query rows of ``raw`` are disjoint."""

    @staticmethod
    def forward(ctx, raw, weight, pos, order, inv, qs, qh, rows, offsets, entries, size):
        ops = _ext.ops()
        updates = ops.gather_rows(raw, None, order)
        conv = ops.conv_fwd(updates, weight, pos)
        query = ops.qconv_fwd(raw, updates, weight[:size], qs, qh)
        ctx.save_for_backward(raw, updates, weight, pos, inv, qs, qh, rows, offsets, entries)
        ctx.size, ctx.n_raw = size, raw.shape[0]
        ctx.mark_non_differentiable(updates)
        return updates, conv, query

    @staticmethod
    def backward(ctx, _d_updates, d_conv, d_query):
        raw, updates, weight, pos, inv, qs, qh, rows, offsets, entries = ctx.saved_tensors
        ops = _ext.ops()
        if d_conv is None:
            d_conv = torch.zeros_like(updates)
        d_upd, dw = ops.conv_bwd(d_conv.contiguous(), updates, weight, pos)
        g = None
        if d_query is not None and qs.numel():
            dwq, g = ops.qconv_bwd_into(d_query.to(torch.bfloat16).contiguous(), raw, updates, weight[:ctx.size], qs,
                                        qh, rows, offsets, entries, d_upd)
            dw[:ctx.size] += dwq
        d_raw = ops.gather_rows_bwd(d_upd, inv, ctx.n_raw, 0)[0]
        if g is not None:
            ops.qconv_raw_grad(g, weight[:ctx.size], qs, d_raw)
        return d_raw, dw.to(weight.dtype), None, None, None, None, None, None, None, None, None


def conv_and_query(raw, weight, plan, size):
    """``(updates, conv, query)`` of a GDN layer: ``updates = raw[plan.content_order]``, the causal
    depthwise conv + SiLU of ``updates`` per document (``weight`` ``[C, K]``), and the query conv of
    the read-only query events over the first ``size`` channels (``query_conv_silu``). CUDA bf16 with
    K = 4 runs the fused node ``_ConvAndQuery``; otherwise the three ops run one by one."""
    from . import gather as GA
    C, K = weight.shape
    fused = (raw.is_cuda and raw.dtype == torch.bfloat16 and K == 4 and size % 8 == 0 and C % 8 == 0
             and raw.stride(-1) == 1 and raw.stride(0) % 8 == 0 and raw.data_ptr() % 16 == 0
             and plan.query_hist_rows is not None and _ext.has("qconv_bwd_into"))
    if fused:
        from .gdn_cuda import _positions
        pos = _positions(tuple(int(b) for b in plan.content_bounds), raw.device)
        if pos.numel() == plan.content_order.numel():
            inv = GA._stacked(plan.content_order_inv)
            return _ConvAndQuery.apply(raw, weight, pos, plan.content_order, inv, plan.query_source,
                                       plan.query_history, plan.query_hist_rows, plan.query_hist_offsets,
                                       plan.query_hist_entries, size)
    updates = GA.rows(raw, plan.content_order, plan.content_order_inv)
    conv = causal_conv_silu(updates, weight, plan.content_bounds)
    query = query_conv_silu(raw, updates, weight[:size], plan)
    return updates, conv, query


def decode_step(state, q, k, v, g, beta):
    """One recurrent step of every head: ``state`` ``[H, Dk, Dv]`` (fp32, in place) takes the write
    ``k [H, Dk]``, ``v [H, Dv]`` with log-decay ``g`` and ``beta`` ``[H]``; the rows of ``q``
    ``[rows, H, Dk]`` read the updated state. q/k are raw (L2-normalised here). Returns fp32
    ``[rows, H, Dv]`` (reference ``ops/gated_delta_net.py:315-352``)."""
    if state.is_cuda and _ext.cuda_kernels_enabled() and _ext.has("gdn_decode_step") and state.shape[1] == 128 \
            and state.shape[2] % 32 == 0 and q.shape[0] <= 4:
        from .gdn_cuda import decode_step as cuda_step
        return cuda_step(state, q, k, v, g, beta)
    ctrl = state.dtype
    qn = R.l2norm(q).to(ctrl) * q.shape[-1] ** -0.5
    kn = R.l2norm(k).to(ctrl)
    state.mul_(g.to(ctrl).exp()[:, None, None])
    residual = v.to(ctrl) - torch.einsum("hkv,hk->hv", state, kn)
    state.add_(kn[:, :, None] * (residual * beta.to(ctrl)[:, None])[:, None, :])
    return torch.einsum("hkv,bhk->bhv", state, qn)


def causal_conv_silu(x, weight, bounds):
    """Causal depthwise conv + SiLU per document over content order; x ``[n, C]``, weight ``[C, K]``."""
    if x.is_cuda and _ext.cuda_kernels_enabled() and hasattr(_ext.ops(), "conv_fwd") and x.dtype == torch.bfloat16:
        from .gdn_cuda import causal_conv_cuda
        return causal_conv_cuda(x, weight, bounds)
    return R.causal_conv_silu(x, weight, bounds)


class _QueryConv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, raw, updates, weight, qs, qh, rows, offsets, entries):
        ctx.save_for_backward(raw, updates, weight, qs, qh, rows, offsets, entries)
        return _ext.ops().qconv_fwd(raw, updates, weight, qs, qh)

    @staticmethod
    def backward(ctx, dy):
        raw, updates, weight, qs, qh, rows, offsets, entries = ctx.saved_tensors
        d_raw, d_upd, dw = _ext.ops().qconv_bwd(dy.to(torch.bfloat16), raw, updates, weight, qs, qh, rows, offsets,
                                                entries)
        return d_raw, d_upd, dw.to(weight.dtype), None, None, None, None, None


def query_conv_silu(raw, updates, weight, plan):
    """Short conv + SiLU of the read-only query events: each query's own projection (``raw`` row
    ``plan.query_source``) plus the last K-1 content inputs of its document (``updates`` rows
    ``plan.query_history``; the index ``len(updates)`` reads zeros). Only the first
    ``weight.shape[0]`` channels of ``raw``/``updates`` are used. Returns ``[nq, channels]``.

    CUDA runs ``qconv_fwd``/``qconv_bwd`` (``csrc/conv.cu``): the backward sums each content row's
    history gradient over the CSR ``plan.query_hist_*`` (deterministic, no atomics).
    """
    size, K = weight.shape
    rows_ok = all(t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 for t in (raw, updates))
    if (raw.is_cuda and raw.dtype == torch.bfloat16 and K == 4 and size % 8 == 0 and rows_ok
            and _ext.has("qconv_fwd") and plan.query_hist_rows is not None):
        return _QueryConv.apply(raw, updates, weight, plan.query_source, plan.query_history, plan.query_hist_rows,
                                plan.query_hist_offsets, plan.query_hist_entries)
    from . import gather as GA
    history = torch.cat((updates[:, :size], updates.new_zeros(1, size)), 0)
    qraw = GA.rows(raw[:, :size], plan.query_source, plan.query_source_inv)
    query = qraw * weight[:, -1].to(qraw.dtype)
    for j in range(K - 1):
        query = query + history.index_select(0, plan.query_history[:, j]) * weight[:, j].to(qraw.dtype)
    if raw.dtype == torch.float64:
        return torch.nn.functional.silu(query)
    return torch.nn.functional.silu(query.float()).to(raw.dtype)
