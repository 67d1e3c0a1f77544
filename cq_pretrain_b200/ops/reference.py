"""Plain-PyTorch definitions of every op (the numerical oracles; CPU and CUDA).

Each function states the math the sm_100a kernels implement. Tests compare kernels against
these in float32/float64. Citations give the reference behaviour each one reproduces.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _f(x):
    """fp32 compute copy (float64 stays float64 so the oracles are exact in double precision)."""
    return x if x.dtype == torch.float64 else x.float()


# ---- normalisation ------------------------------------------------------------------------
def rms_norm(x, weight, eps, offset=True):
    """Qwen RMSNorm ``x * rsqrt(mean x^2 + eps) * (1 + w)`` computed in fp32 (reference ``backbone_qwen35.py:13-28``)."""
    w = (1 + _f(weight)) if offset else _f(weight)
    xf = _f(x)
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w).to(x.dtype)


def gated_rms_norm(x, z, weight, eps):
    """GDN output norm ``rms(x) * w * silu(z)`` per head (reference ``backbone_qwen35.py:101-114``)."""
    xf = _f(x)
    normed = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)).to(x.dtype)
    return (normed * weight.to(x.dtype) * F.silu(_f(z)).to(x.dtype)).to(x.dtype)


def layer_norm_modulate(x, scale, shift, eps):
    """Wan adaLN: ``LayerNorm(x) (fp32, no affine) * (1 + scale) + shift`` (reference ``ops/torchair.py:8-12``)."""
    normed = F.layer_norm(_f(x), (x.shape[-1],), eps=eps)
    return normed * (1 + _f(scale)) + _f(shift)


def gated_add(x, branch, gate):
    """FP32 gated residual ``x + gate * branch``."""
    return _f(x) + _f(gate) * _f(branch)


# ---- activations ---------------------------------------------------------------------------
def swiglu(x):
    gate, up = x.chunk(2, -1)
    return (F.silu(_f(gate)) * _f(up)).to(x.dtype)


def gelu_tanh(x):
    return F.gelu(_f(x), approximate="tanh").to(x.dtype)


# ---- rotary -------------------------------------------------------------------------------
def rotary_half(x, cos, sin, dim):
    """Rotate-half RoPE on the first ``dim`` channels of each head; x ``[rows, heads, hd]``, cos ``[rows, dim]``."""
    rot, rest = _f(x[..., :dim]), x[..., dim:]
    c, s = cos[:, None, :].to(rot.dtype), sin[:, None, :].to(rot.dtype)
    a, b = rot.chunk(2, -1)
    out = rot * c + torch.cat((-b, a), -1) * s
    return torch.cat((out.to(x.dtype), rest), -1)


def rotary_pairs(x, cos, sin):
    """Wan complex-pair RoPE: pairs (x[2i], x[2i+1]) rotated by angle i; cos ``[rows, hd/2]``."""
    real, imag = _f(x).unflatten(-1, (-1, 2)).unbind(-1)
    c, s = cos[:, None, :].to(real.dtype), sin[:, None, :].to(real.dtype)
    return torch.stack((real * c - imag * s, imag * c + real * s), -1).flatten(-2).to(x.dtype)


# ---- attention ------------------------------------------------------------------------------
def range_attention(q, k, v, kstart, kend, scale=None, tile=2048):
    """Softmax attention where row r sees keys [kstart[r], kend[r]); empty rows output 0.

    q ``[rows, Hq, D]``, k/v ``[keys, Hkv, D]`` (GQA: Hq multiple of Hkv). This is the CQ mask of
    the reference (``ops/attention_layout.py:69-102``) expressed as per-row key ranges.
    """
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    rep = q.shape[1] // k.shape[1]
    kk = k.repeat_interleave(rep, 1) if rep > 1 else k
    vv = v.repeat_interleave(rep, 1) if rep > 1 else v
    keys = torch.arange(k.shape[0], device=q.device)
    out = torch.empty_like(q)
    for r0 in range(0, q.shape[0], tile):
        r1 = min(r0 + tile, q.shape[0])
        ks, ke = kstart[r0:r1].long(), kend[r0:r1].long()
        valid = ke > ks
        if not bool(valid.any()):
            out[r0:r1] = 0
            continue
        lo, hi = int(ks[valid].min()), int(ke[valid].max())
        kv_keys = keys[lo:hi]
        allowed = (kv_keys[None] >= ks[:, None]) & (kv_keys[None] < ke[:, None])
        allowed[~valid, 0] = True
        res = F.scaled_dot_product_attention(q[r0:r1].transpose(0, 1)[None], kk[lo:hi].transpose(0, 1)[None],
                                             vv[lo:hi].transpose(0, 1)[None], attn_mask=allowed[None, None],
                                             scale=scale)[0].transpose(0, 1)
        out[r0:r1] = res * valid[:, None, None].to(res.dtype)
    return out


def varlen_attention(q, k, v, q_ends, k_ends, scale=None):
    """Non-causal attention inside each packed sample; q ``[Lq, H, D]``, k/v ``[Lk, H, D]``; ends cumulative."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    out = []
    qa = ka = 0
    for qb, kb in zip(q_ends, k_ends):
        if kb == ka:
            out.append(q.new_zeros(qb - qa, q.shape[1], v.shape[2]))
            qa = qb
            continue
        a, b, c = (t.transpose(0, 1)[None] for t in (q[qa:qb], k[ka:kb], v[ka:kb]))
        out.append(F.scaled_dot_product_attention(a, b, c, scale=scale)[0].transpose(0, 1))
        qa, ka = qb, kb
    return torch.cat(out) if out else q.new_zeros(q.shape)


# ---- gated delta rule ---------------------------------------------------------------------
def l2norm(x, eps=1e-6):
    xf = _f(x)
    return xf * torch.rsqrt(xf.square().sum(-1, keepdim=True) + eps)


def recurrent_gated_delta(q, k, v, g, beta, bounds, initial=None, final=False):
    """Token-by-token gated delta rule (the differentiable oracle, reference ``backbone_qwen35.py:56-73``).

    q, k ``[E, H, Dk]``; v ``[E, H, Dv]``; g, beta ``[E, H]``; ``bounds`` document boundaries.
    q/k are L2-normalised here (q also scaled by Dk^-0.5). Per step:
    ``S = e^g S;  S += k (beta (v - S^T k))^T;  o = S^T q``.
    """
    q = l2norm(q) * q.shape[-1] ** -0.5
    k = l2norm(k)
    v = _f(v)
    outputs, states = [], []
    for d, (a, b) in enumerate(zip(bounds, bounds[1:])):
        state = (q.new_zeros(q.shape[1], q.shape[2], v.shape[2]) if initial is None else _f(initial[d]))
        for i in range(a, b):
            state = state * _f(g[i]).exp()[:, None, None]
            residual = v[i] - torch.einsum("hkv,hk->hv", state, k[i])
            state = state + k[i][:, :, None] * (residual * _f(beta[i])[:, None])[:, None, :]
            outputs.append(torch.einsum("hkv,hk->hv", state, q[i]))
        states.append(state)
    out = torch.stack(outputs) if outputs else v.new_zeros(0, v.shape[1], v.shape[2])
    return (out, torch.stack(states)) if final else out


def chunk_layout(bounds, chunk):
    """Map events of each document into zero-padded chunks: (gather index [Nc*C], chunks per doc, doc of chunk)."""
    index, per_doc = [], []
    for a, b in zip(bounds, bounds[1:]):
        n = b - a
        nchunks = max(1, -(-n // chunk)) if n else 0
        rows = list(range(a, b)) + [-1] * (nchunks * chunk - n)
        index.extend(rows)
        per_doc.append(nchunks)
    return index, per_doc


def chunk_gated_delta(q, k, v, g, beta, bounds, chunk=64, initial=None, final=False):
    """Chunked (WY) gated delta rule, exact up to rounding with :func:`recurrent_gated_delta`.

    Per chunk with inclusive cumulative log-decay ``b`` and incoming state ``S0``:
    ``A = tril(beta_i e^{b_i-b_j} k_i.k_j, -1)``, ``T = (I + A)^-1``,
    ``W = T diag(beta e^b) K``, ``U = T diag(beta) V``, ``D = U - W S0``,
    ``O = diag(e^b) Q S0 + (tril(Q K^T e^{b_i-b_j})) D``, ``S1 = e^{b_C} S0 + (K e^{b_C-b})^T D``.
    """
    dtype = torch.float64 if q.dtype == torch.float64 else torch.float32
    E, H, Dk = q.shape
    Dv = v.shape[-1]
    qn = (l2norm(q) * Dk ** -0.5).to(dtype)
    kn = l2norm(k).to(dtype)
    index, per_doc = chunk_layout(bounds, chunk)
    idx = torch.tensor(index, dtype=torch.long, device=q.device)
    pad = idx < 0
    safe = idx.clamp_min(0)

    def gather(t):
        x = t.to(dtype).index_select(0, safe)
        return x.masked_fill(pad.view(-1, *([1] * (x.dim() - 1))), 0)

    Nc = len(index) // chunk
    Q = gather(qn).view(Nc, chunk, H, Dk).transpose(1, 2)          # [Nc, H, C, Dk]
    K = gather(kn).view(Nc, chunk, H, Dk).transpose(1, 2)
    V = gather(v).view(Nc, chunk, H, Dv).transpose(1, 2)
    G = gather(g).view(Nc, chunk, H).transpose(1, 2)                # [Nc, H, C]
    B = gather(beta).view(Nc, chunk, H).transpose(1, 2)
    b = G.cumsum(-1)
    diff = b[..., :, None] - b[..., None, :]
    strict = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril(-1)
    incl = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril()
    decay_strict = torch.where(strict, diff, torch.full_like(diff, -math.inf)).exp()
    decay_incl = torch.where(incl, diff, torch.full_like(diff, -math.inf)).exp()
    A = (K @ K.transpose(-1, -2)) * decay_strict * B[..., :, None]
    eye = torch.eye(chunk, dtype=dtype, device=q.device)
    T = torch.linalg.solve_triangular(eye + A, eye.expand_as(A), upper=False, unitriangular=True)
    W = T @ (K * (B * b.exp())[..., None])
    U = T @ (V * B[..., None])
    P = (Q @ K.transpose(-1, -2)) * decay_incl
    Qd = Q * b.exp()[..., None]
    Kd = K * (b[..., -1:] - b).exp()[..., None]
    last = b[..., -1].exp()
    # Sequential pass over chunk positions; all documents advance together.
    starts = [0]
    for n in per_doc:
        starts.append(starts[-1] + n)
    ndocs = len(per_doc)
    state = [(q.new_zeros(H, Dk, Dv, dtype=dtype) if initial is None else initial[d].to(dtype)) for d in range(ndocs)]
    outs = [None] * Nc
    for c in range(max(per_doc, default=0)):
        docs = [d for d in range(ndocs) if per_doc[d] > c]
        ids = torch.tensor([starts[d] + c for d in docs], device=q.device)
        S0 = torch.stack([state[d] for d in docs])
        D = U[ids] - W[ids] @ S0
        O = Qd[ids] @ S0 + P[ids] @ D
        S1 = last[ids][..., None, None] * S0 + Kd[ids].transpose(-1, -2) @ D
        for j, d in enumerate(docs):
            outs[starts[d] + c] = O[j]
            state[d] = S1[j]
    O = torch.stack(outs).transpose(1, 2).reshape(Nc * chunk, H, Dv)
    keep = (~pad).nonzero().flatten()
    out = O.index_select(0, keep)
    if final:
        return out, torch.stack(state)
    return out


def causal_conv_silu(x, weight, bounds):
    """Depthwise causal conv (kernel K) + SiLU over each document; x ``[n, C]``, weight ``[C, K]``."""
    n, K = x.shape[0], weight.shape[-1]
    pos = torch.empty(n, dtype=torch.long, device=x.device)
    for a, b in zip(bounds, bounds[1:]):
        pos[a:b] = torch.arange(b - a, device=x.device)
    xf = _f(x)
    y = xf * _f(weight[:, K - 1])
    for i in range(K - 1):
        shift = K - 1 - i
        shifted = torch.zeros_like(xf)
        shifted[shift:] = xf[:-shift] if shift < n else shifted[shift:]
        shifted = shifted * (pos >= shift)[:, None]
        y = y + shifted * _f(weight[:, i])
    return F.silu(y).to(x.dtype)


# ---- loss ---------------------------------------------------------------------------------
def cross_entropy_rows(hidden, weight, targets):
    logits = _f(hidden) @ _f(weight).T
    return F.cross_entropy(logits, targets, reduction="none")
