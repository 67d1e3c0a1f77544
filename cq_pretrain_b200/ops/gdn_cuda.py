"""CUDA path of the chunked gated delta rule.

Chunk-local work (parallel over every chunk and head) runs in ``csrc/gdn_chunk.cu``: the WY
factors of the forward, and one fused kernel for the whole chunk-local backward. The two
sequential passes over the chunks of each document, the forward state recurrence and the
backward state-gradient recurrence, run in ``csrc/gdn.cu``. ``chunk_gather``/``chunk_scatter``
(``csrc/conv.cu``) move events into the zero-padded chunk layout with the q/k L2 norm fused.
Per chunk (cumulative log-decay ``b``, ``E_ij = e^{b_i-b_j}``):

    A = tril(beta_i E_ij k_i.k_j, -1)     T = (I + A)^-1
    W = T diag(beta e^b) K                U = T diag(beta) V
    P = tril(Q K^T * E)                   Qd = diag(e^b) Q     Kt = diag(e^{b_C - b}) K
    gamma = e^{b_C}
    kernel:  D = U - W S;  O = Qd S + P D;  S <- gamma S + Kt^T D
"""

from __future__ import annotations

import math
import os
from functools import lru_cache

import torch

from . import _ext
from . import reference as R

CHUNK = 64


@lru_cache(maxsize=64)
def _layout_host(bounds, chunk):
    index, per_doc = R.chunk_layout(bounds, chunk)
    starts, s = [], 0
    for n in per_doc:
        starts.append(s)
        s += n
    return tuple(index), tuple(starts), tuple(per_doc)


_DEVICE_LAYOUTS: dict = {}


def _layout(bounds, chunk, device):
    """Device chunk layout: (slot -> event index or -1, pad mask, event -> slot, doc chunk starts/counts, Nc)."""
    key = (bounds, chunk, str(device))
    hit = _DEVICE_LAYOUTS.get(key)
    if hit is None:
        index, starts, counts = _layout_host(bounds, chunk)
        idx = torch.tensor(index, dtype=torch.long)
        pad = idx < 0
        keep = (~pad).nonzero().flatten()
        hit = (idx.to(device), pad.to(device), keep.to(device),
               torch.tensor(starts, dtype=torch.int32).to(device), torch.tensor(counts, dtype=torch.int32).to(device),
               len(index) // chunk)
        if len(_DEVICE_LAYOUTS) > 64:
            _DEVICE_LAYOUTS.clear()
        _DEVICE_LAYOUTS[key] = hit
    return hit


def _factors(Q, K, V, G, B, chunk):
    """WY factors of every chunk (no autograd). Q, K, V bf16 ``[Nc,H,C,D]``; G, B fp32 ``[Nc,H,C]``."""
    bf = torch.bfloat16
    b = G.cumsum(-1)
    diff = b[..., :, None] - b[..., None, :]
    tri = torch.ones(chunk, chunk, dtype=torch.bool, device=Q.device)
    neg = torch.full((), -math.inf, device=Q.device)
    e_strict = torch.where(tri.tril(-1), diff, neg).exp_()
    e_incl = torch.where(tri.tril(), diff, neg).exp_()
    del diff
    KK = torch.matmul(K, K.transpose(-1, -2)).float()
    A = KK * e_strict
    A.mul_(B[..., :, None])
    eye = torch.eye(chunk, dtype=torch.float32, device=Q.device)
    T = torch.linalg.solve_triangular(eye + A, eye.expand_as(A), upper=False, unitriangular=True)
    Tb = T.to(bf)
    eb = b.exp()
    Kw = (K * (B * eb)[..., None].to(bf))
    Vb = (V * B[..., None].to(bf))
    W = torch.matmul(Tb, Kw)
    U = torch.matmul(Tb, Vb)
    QK = torch.matmul(Q, K.transpose(-1, -2)).float()
    P = (QK * e_incl).to(bf)
    Qd = Q * eb[..., None].to(bf)
    kdec = (b[..., -1:] - b).exp()
    Kt = K * kdec[..., None].to(bf)
    gamma = b[..., -1].exp().contiguous()
    return dict(b=b, eb=eb, kdec=kdec, e_strict=e_strict, e_incl=e_incl, KK=KK, A=A, T=T, Tb=Tb, Kw=Kw, Vb=Vb,
                W=W.contiguous(), U=U.contiguous(), P=P.contiguous(), QK=QK, Qd=Qd.contiguous(), Kt=Kt.contiguous(),
                gamma=gamma)


# The fused chunk backward has a tcgen05 form (``gdn_chunk_bwd_tc_kernel``: bf16 states by TMA); it is
# correct but slower than the mma.sync form at one unit per SM (its per-unit chain of dependent MMA
# groups is latency-bound), so the mma.sync form is the default and CQB_GDN_CHUNK_TC=1 selects it.
_CHUNK_TC = os.environ.get("CQB_GDN_CHUNK_TC", "0") == "1"


class _GatedDelta(torch.autograd.Function):
    """q, k, v ``[E,H,D]`` (bf16), g, beta ``[E,H]`` fp32 -> o ``[E,H,Dv]``; analytic chunked backward."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, layout, chunk):
        idx, pad, keep, start, count, Nc = layout
        E, H, Dk = q.shape
        ops = _ext.ops()
        Q, rq = ops.chunk_gather(q, idx, Nc, True, Dk ** -0.5)
        K, rk = ops.chunk_gather(k, idx, Nc, True, 1.0)
        V = ops.chunk_gather(v, idx, Nc, False, 1.0)[0]
        G, B = _to_chunks((g.float(), beta.float()), idx, pad, Nc, chunk, H)
        W, U, P, Qd, Kt, gamma = ops.gdn_prep(Q, K, V, G, B)
        O, S = ops.gdn_fwd(W, U, P, Qd, Kt, gamma, start, count, want_final=False)
        # the backward reuses the chunk-layout inputs and the recurrence factors instead of
        # gathering and recomputing them (about 0.45 GB per layer at 8K tokens and 16 heads)
        ctx.save_for_backward(q, k, v, rq, rk, S, Q, K, V, G, B, W, P, Qd, Kt, gamma)
        ctx.layout, ctx.chunk = layout, chunk
        ctx.g_dtype, ctx.beta_dtype = g.dtype, beta.dtype
        return ops.chunk_scatter(O, keep, O, O, False, 1.0)

    @staticmethod
    def backward(ctx, dout):
        q, k, v, rq, rk, S, Q, K, V, G, B, W, P, Qd, Kt, gamma = ctx.saved_tensors
        idx, pad, keep, start, count, Nc = ctx.layout
        chunk = ctx.chunk
        E, H, Dk = q.shape
        ops = _ext.ops()
        dO = ops.chunk_gather(dout.to(torch.bfloat16).contiguous(), idx, Nc, False, 1.0)[0]
        dS = ops.gdn_bwd(dO, W, P, Qd, Kt, gamma, start, count)
        del W, P, Qd, Kt
        if _CHUNK_TC:   # the tcgen05 chunk backward takes bf16 states and dgamma = <S, dS>
            dgamma = (S * dS).sum((-1, -2))
            dQ, dK, dV, dG, dB = ops.gdn_chunk_bwd(Q, K, V, dO, G, B, S.to(torch.bfloat16), dS.to(torch.bfloat16),
                                                   dgamma)
        else:
            dQ, dK, dV, dG, dB = ops.gdn_chunk_bwd(Q, K, V, dO, G, B, S, dS)
        del dS

        def back(t):
            return t.transpose(1, 2).reshape(Nc * chunk, H).index_select(0, keep)

        dq = ops.chunk_scatter(dQ, keep, q, rq, True, Dk ** -0.5)
        dk = ops.chunk_scatter(dK, keep, k, rk, True, 1.0)
        dv = ops.chunk_scatter(dV, keep, v, rk, False, 1.0)
        return dq, dk, dv, back(dG).to(ctx.g_dtype), back(dB).to(ctx.beta_dtype), None, None


def chunk_backward_reference(Q, K, V, dO, G, B, S, dS, chunk=CHUNK):
    """PyTorch form of the fused chunk backward (``gdn_chunk_bwd``), used to test the kernel.

    Inputs in chunk layout (``[Nc, H, C, D]`` bf16, ``[Nc, H, C]`` fp32, states fp32); returns
    ``dQ, dK, dV`` (fp32) and ``dG, dBeta`` of every chunk.
    """
    bf = torch.bfloat16
    f = _factors(Q, K, V, G, B, chunk)
    Sb, dSb = S.to(bf), dS.to(bf)
    Delta = (f["U"].float() - torch.matmul(f["W"], Sb).float()).to(bf)
    dDelta = (torch.matmul(f["P"].transpose(-1, -2), dO).float() + torch.matmul(f["Kt"], dSb).float()).to(bf)
    dW = -torch.matmul(dDelta, Sb.transpose(-1, -2)).float()
    dQd = torch.matmul(dO, Sb.transpose(-1, -2)).float()
    dP = torch.matmul(dO, Delta.transpose(-1, -2)).float()
    dKt = torch.matmul(Delta, dSb.transpose(-1, -2)).float()
    dgamma = (S * dS).sum((-1, -2))
    dU = dDelta.float()
    eb, kdec = f["eb"], f["kdec"]
    # Qd = e^b Q
    dQ = dQd * eb[..., None]
    db = (dQd * f["Qd"].float()).sum(-1)
    # P = (Q K^T) * E_incl
    dPm = dP * f["e_incl"]
    dQ += torch.matmul(dPm.to(bf), K).float()
    dK = torch.matmul(dPm.transpose(-1, -2).to(bf), Q).float()
    t = dP * (f["QK"] * f["e_incl"])
    db += t.sum(-1) - t.sum(-2)
    # Kt = e^{b_C - b} K
    dK += dKt * kdec[..., None]
    rkt = (dKt * f["Kt"].float()).sum(-1)
    db -= rkt
    dbC = rkt.sum(-1) + dgamma * f["gamma"]
    # U = T Vb, W = T Kw
    Tb = f["Tb"]
    dT = (torch.matmul(dU.to(bf), f["Vb"].transpose(-1, -2)).float()
          + torch.matmul(dW.to(bf), f["Kw"].transpose(-1, -2)).float())
    dVb = torch.matmul(Tb.transpose(-1, -2), dU.to(bf)).float()
    dKw = torch.matmul(Tb.transpose(-1, -2), dW.to(bf)).float()
    dV = dVb * B[..., None]
    dbeta = (dVb * V.float()).sum(-1)
    sw = (dKw * K.float()).sum(-1)
    dbeta += sw * eb
    db += sw * eb * B
    dK += dKw * (B * eb)[..., None]
    # T = (I + A)^-1  ->  dA = -T^T dT T^T (strict lower part)
    T = f["T"]
    dA = -torch.matmul(torch.matmul(T.transpose(-1, -2), dT), T.transpose(-1, -2))
    dA = dA * torch.ones(chunk, chunk, dtype=torch.bool, device=Q.device).tril(-1)
    tA = dA * f["A"]
    dbeta += (dA * f["KK"] * f["e_strict"]).sum(-1)
    db += tA.sum(-1) - tA.sum(-2)
    dKK = dA * f["e_strict"] * B[..., :, None]
    dK += torch.matmul((dKK + dKK.transpose(-1, -2)).to(bf), K).float()
    # b = cumsum(g) within the chunk: dg_i = sum_{j >= i} db_j ; b_C also feeds gamma and Kt
    db[..., -1] += dbC
    dG = db.flip(-1).cumsum(-1).flip(-1)
    return dQ, dK, dV, dG, dbeta


def _to_chunks(tensors, idx, pad, Nc, chunk, H):
    """Per-event ``[E, H(, D)]`` tensors -> zero-padded chunk layout ``[Nc, H, C(, D)]``."""
    idx = idx.clamp_min(0)
    out = []
    for t in tensors:
        x = t.index_select(0, idx)
        x = x.masked_fill(pad.view(-1, *([1] * (x.dim() - 1))), 0)
        if x.dim() == 3:
            out.append(x.view(Nc, chunk, H, x.shape[-1]).transpose(1, 2).contiguous())
        else:
            out.append(x.view(Nc, chunk, H).transpose(1, 2).contiguous())
    return out


def gated_delta_cuda(q, k, v, g, beta, bounds, chunk=CHUNK, final=False):
    """Event-ordered inputs -> event-ordered outputs ``[E, H, Dv]`` (bf16). With ``final`` (prefill,
    no autograd) also the fp32 state after each document ``[docs, H, Dk, Dv]``, produced by the
    forward recurrence kernel itself."""
    E, H, Dk = q.shape
    Dv = v.shape[-1]
    if Dk != 128 or Dv != 128 or chunk != CHUNK:
        if final:
            y, state = R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk, final=True)
            return y.to(v.dtype), state
        return R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk).to(v.dtype)
    layout = _layout(tuple(int(x) for x in bounds), chunk, q.device)
    bf = torch.bfloat16
    if final:
        return _prefill(q.to(bf).contiguous(), k.to(bf).contiguous(), v.to(bf).contiguous(), g, beta, layout, chunk)
    return _GatedDelta.apply(q.to(bf).contiguous(), k.to(bf).contiguous(), v.to(bf).contiguous(), g, beta, layout,
                             chunk)


@torch.no_grad()
def _prefill(q, k, v, g, beta, layout, chunk):
    idx, pad, keep, start, count, Nc = layout
    E, H, Dk = q.shape
    ops = _ext.ops()
    Q = ops.chunk_gather(q, idx, Nc, True, Dk ** -0.5)[0]
    K = ops.chunk_gather(k, idx, Nc, True, 1.0)[0]
    V = ops.chunk_gather(v, idx, Nc, False, 1.0)[0]
    G, B = _to_chunks((g.float(), beta.float()), idx, pad, Nc, chunk, H)
    W, U, P, Qd, Kt, gamma = ops.gdn_prep(Q, K, V, G, B)
    O, _, state = ops.gdn_fwd(W, U, P, Qd, Kt, gamma, start, count, want_final=True)
    return ops.chunk_scatter(O, keep, O, O, False, 1.0), state


def decode_step(state, q, k, v, g, beta):
    """One fused recurrent step for all heads (``csrc/gdn_decode.cu``): ``state`` fp32 ``[H, Dk, Dv]``
    updated in place by the write of ``k``/``v`` (raw, L2-normalised inside), then every row of
    ``q`` ``[rows, H, Dk]`` reads it. Returns fp32 ``[rows, H, Dv]``."""
    f = torch.float32
    out = torch.empty(q.shape[0], state.shape[0], state.shape[2], dtype=f, device=state.device)
    _ext.ops().gdn_decode_step(state, q.to(f).contiguous(), k.to(f).contiguous(), v.to(f).contiguous(),
                               g.to(f).contiguous(), beta.to(f).contiguous(), out)
    return out


_POSITIONS: dict = {}


def _positions(bounds, device):
    """int32 index of each row inside its document (cached per packing)."""
    key = (bounds, str(device))
    hit = _POSITIONS.get(key)
    if hit is None:
        pos = torch.empty(bounds[-1] if bounds else 0, dtype=torch.int32)
        for a, b in zip(bounds, bounds[1:]):
            pos[a:b] = torch.arange(b - a, dtype=torch.int32)
        hit = pos.to(device)
        if len(_POSITIONS) > 64:
            _POSITIONS.clear()
        _POSITIONS[key] = hit
    return hit


class _CausalConv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, pos):
        ctx.save_for_backward(x, weight, pos)
        return _ext.ops().conv_fwd(x, weight, pos)

    @staticmethod
    def backward(ctx, dy):
        x, weight, pos = ctx.saved_tensors
        dx, dw = _ext.ops().conv_bwd(dy.contiguous(), x, weight, pos)
        return dx, dw.to(weight.dtype), None


def causal_conv_cuda(x, weight, bounds):
    """Causal depthwise conv (kernel 4) + SiLU per document in ``csrc/conv.cu``; other kernels fall back."""
    if weight.shape[-1] != 4 or x.shape[-1] % 8:
        return R.causal_conv_silu(x, weight, bounds)
    pos = _positions(tuple(int(b) for b in bounds), x.device)
    if pos.numel() != x.shape[0]:
        raise ValueError(f"document bounds cover {pos.numel()} rows, x has {x.shape[0]}")
    return _CausalConv.apply(x.contiguous(), weight, pos)
