"""CUDA path of the chunked gated delta rule.

Chunk-local WY factors (parallel over every chunk and head) are batched tensor-core GEMMs and
a batched triangular solve; the two sequential passes over the chunks of each document, the
forward state recurrence and the backward state-gradient recurrence, run in the hand-written
sm_100a kernels of ``csrc/gdn.cu``. Per chunk (cumulative log-decay ``b``, ``E_ij = e^{b_i-b_j}``):

    A = tril(beta_i E_ij k_i.k_j, -1)     T = (I + A)^-1
    W = T diag(beta e^b) K                U = T diag(beta) V
    P = tril(Q K^T * E)                   Qd = diag(e^b) Q     Kt = diag(e^{b_C - b}) K
    gamma = e^{b_C}
    kernel:  D = U - W S;  O = Qd S + P D;  S <- gamma S + Kt^T D
"""

from __future__ import annotations

import math
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
    key = (bounds, chunk, str(device))
    hit = _DEVICE_LAYOUTS.get(key)
    if hit is None:
        index, starts, counts = _layout_host(bounds, chunk)
        idx = torch.tensor(index, dtype=torch.long)
        pad = idx < 0
        keep = (~pad).nonzero().flatten()
        hit = (idx.clamp_min(0).to(device), pad.to(device), keep.to(device),
               torch.tensor(starts, dtype=torch.int32).to(device), torch.tensor(counts, dtype=torch.int32).to(device),
               len(index) // chunk)
        if len(_DEVICE_LAYOUTS) > 64:
            _DEVICE_LAYOUTS.clear()
        _DEVICE_LAYOUTS[key] = hit
    return hit


class _Recurrence(torch.autograd.Function):
    @staticmethod
    def forward(ctx, W, U, P, Qd, Kt, gamma, start, count):
        O, S = _ext.ops().gdn_fwd(W, U, P, Qd, Kt, gamma, start, count)
        ctx.save_for_backward(W, U, P, Qd, Kt, gamma, start, count, S)
        return O

    @staticmethod
    def backward(ctx, dO):
        W, U, P, Qd, Kt, gamma, start, count, S = ctx.saved_tensors
        dO = dO.contiguous().to(torch.bfloat16)
        dS = _ext.ops().gdn_bwd(dO, W, P, Qd, Kt, gamma, start, count)
        Sb, dSb = S.to(torch.bfloat16), dS.to(torch.bfloat16)
        Delta = (U.float() - torch.matmul(W, Sb).float()).to(torch.bfloat16)
        dDelta = (torch.matmul(P.transpose(-1, -2), dO).float() + torch.matmul(Kt, dSb).float()).to(torch.bfloat16)
        dW = -torch.matmul(dDelta, Sb.transpose(-1, -2))
        dQd = torch.matmul(dO, Sb.transpose(-1, -2))
        dP = torch.matmul(dO, Delta.transpose(-1, -2))
        dKt = torch.matmul(Delta, dSb.transpose(-1, -2))
        dgamma = (S * dS).sum((-1, -2))
        return dW, dDelta, dP, dQd, dKt, dgamma, None, None


def gated_delta_cuda(q, k, v, g, beta, bounds, chunk=CHUNK):
    """Event-ordered inputs -> event-ordered outputs ``[E, H, Dv]`` (bf16)."""
    E, H, Dk = q.shape
    Dv = v.shape[-1]
    if Dk != 128 or Dv % 64 or chunk != CHUNK:
        return R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk).to(v.dtype)
    idx, pad, keep, start, count, Nc = _layout(tuple(int(x) for x in bounds), chunk, q.device)
    bf = torch.bfloat16
    qn = (R.l2norm(q) * Dk ** -0.5).to(bf)
    kn = R.l2norm(k).to(bf)
    padc = pad.view(-1, 1, 1)

    def gather(t):
        x = t.index_select(0, idx)
        return x.masked_fill(padc if x.dim() == 3 else pad.view(-1, 1), 0)

    Q = gather(qn).view(Nc, chunk, H, Dk).transpose(1, 2)
    K = gather(kn).view(Nc, chunk, H, Dk).transpose(1, 2)
    V = gather(v.to(bf)).view(Nc, chunk, H, Dv).transpose(1, 2)
    G = gather(g.float()).view(Nc, chunk, H).transpose(1, 2)
    B = gather(beta.float()).view(Nc, chunk, H).transpose(1, 2)
    b = G.cumsum(-1)
    diff = b[..., :, None] - b[..., None, :]
    tri = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device)
    strict, incl = tri.tril(-1), tri.tril()
    neg = torch.full_like(diff, -math.inf)
    e_strict = torch.where(strict, diff, neg).exp()
    e_incl = torch.where(incl, diff, neg).exp()
    KK = torch.matmul(K, K.transpose(-1, -2)).float()
    A = KK * e_strict * B[..., :, None]
    eye = torch.eye(chunk, dtype=torch.float32, device=q.device)
    T = torch.linalg.solve_triangular(eye + A, eye.expand_as(A), upper=False, unitriangular=True).to(bf)
    eb = b.exp()
    Wf = torch.matmul(T, (K * (B * eb)[..., None].to(bf)).to(bf))
    Uf = torch.matmul(T, (V * B[..., None].to(bf)).to(bf))
    Pf = (torch.matmul(Q, K.transpose(-1, -2)).float() * e_incl).to(bf)
    Qd = (Q * eb[..., None].to(bf)).to(bf)
    Kt = (K * (b[..., -1:] - b).exp()[..., None].to(bf)).to(bf)
    gamma = b[..., -1].exp().contiguous()
    O = _Recurrence.apply(Wf.contiguous(), Uf.contiguous(), Pf.contiguous(), Qd.contiguous(), Kt.contiguous(),
                          gamma, start, count)
    out = O.transpose(1, 2).reshape(Nc * chunk, H, Dv)
    return out.index_select(0, keep)


def causal_conv_cuda(x, weight, bounds):
    return R.causal_conv_silu(x, weight, bounds)
