"""Numerical self-check of the in-kernel TP collectives against NCCL on the live process group.

``fused_vs_nccl()`` runs each fused path once on small random operands and returns its maximum
relative error against the NCCL + GEMM composition, reduced with MAX over all ranks:

* ``allgather_gemm``: all-gather -> GEMM (column-parallel forward);
* ``gemm_reducescatter``: GEMM -> reduce-scatter with the owner-added bias (row-parallel forward);
* ``pair_reducescatter``: the input gradient of two column-parallel projections of one gathered
  input, ``reduce_scatter(dY1 W1 + pad(dY2) W2)``;
* ``allgather_gemm_mn``: ``all_gather(dY) @ W`` (row-parallel input gradient);
* ``tp_rmsnorm``: Wan's full-width RMSNorm with the per-row sums exchanged in-kernel;
* ``ce_exchange``: the vocabulary-parallel (max, sum exp, target logit) exchange.

Every rank issues the same collectives in the same order. Returns ``{}`` without the workspace.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext, gemm
from . import fused
from . import state as ps
from . import symmetric


def _rel(a, b):
    b = b.float()
    return float((a.float() - b).abs().max() / b.abs().max().clamp_min(1e-12))


def fused_vs_nccl(seed=0):
    ws = symmetric.workspace()
    if ws is None:
        return {}
    st = ps.state()
    tp, dev = st.tp, st.device
    gen = torch.Generator(device=dev).manual_seed(seed + 17 * st.tp_rank)

    def randn(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=gen) * scale).to(torch.bfloat16)

    err = {}
    x, w = randn(256, 512), randn(384, 512, scale=0.05)
    y, _ = ws.gather_linear(x, w)
    err["allgather_gemm"] = _rel(y, gemm.linear(fused.gather_rows_raw(x), w))
    xf, w2, bias = randn(256 * tp, 256), randn(512, 256, scale=0.05), randn(512)
    z = ws.linear_scatter(xf, w2, bias)
    err["gemm_reducescatter"] = _rel(z, fused.scatter_rows_raw(gemm.linear(xf, w2)).float() + bias.float())
    dy, w3 = randn(256 * tp, 384), randn(384, 512, scale=0.05)
    dy2, w4 = randn(256 * tp - 72, 160), randn(160, 512, scale=0.05)
    full = gemm.matmul_nn(dy, w3).float()
    full[: dy2.shape[0]] += gemm.matmul_nn(dy2, w4).float()
    err["pair_reducescatter"] = _rel(ws.matmul_scatter(dy, w3, dy2, w4), fused.scatter_rows_raw(full))
    dyl, w5 = randn(256, 384), randn(384, 320, scale=0.05)
    g, _ = ws.gather_matmul(dyl, w5)
    err["allgather_gemm_mn"] = _rel(g, gemm.matmul_nn(fused.gather_rows_raw(dyl), w5))
    xq = randn(1000, 384)
    wq = 1 + 0.1 * torch.randn(384, device=dev, generator=gen)
    yq, _ = ws.rms_forward(xq, wq.contiguous(), 384 * tp, 1e-6)
    sq = xq.float().square().sum(-1, keepdim=True)
    dist.all_reduce(sq, group=st.tp_group)
    err["tp_rmsnorm"] = _rel(yq, xq.float() * torch.rsqrt(sq / (384 * tp) + 1e-6) * wq)
    if ws.supports_ce(448):
        from ..ops.cross_entropy import _stats_combine
        rows, vocab = 448, 1024 * tp
        hid = randn(rows, 256)   # the combine is checked on whatever per-rank partials each rank holds
        tg = torch.randint(0, vocab, (rows,), device=dev, generator=torch.Generator(device=dev).manual_seed(seed))
        wv = randn(vocab // tp, 256, scale=0.05)
        lo = st.tp_rank * (vocab // tp)
        ops = _ext.ops()
        lse_f, tgt_f = ws.ce_combine(*ops.ce_partials(hid, wv, tg, lo))
        mx, tgt_n, se = _stats_combine(*ops.ce_stats(hid, wv, tg, lo), st.tp_group)
        err["ce_exchange"] = max(_rel(lse_f, mx + torch.log(se)), _rel(tgt_f, tgt_n))
    names = sorted(err)
    vals = torch.tensor([err[k] for k in names], dtype=torch.float64, device=dev)
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    status = symmetric.status()
    out = {k: float(v) for k, v in zip(names, vals.tolist())}
    out["status"] = status
    return out
