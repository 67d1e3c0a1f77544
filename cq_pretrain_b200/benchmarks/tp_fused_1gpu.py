"""The fused TP GEMM kernels of rank 0 of a TP = 2 group, emulated on one GPU (for ncu).

``python -m cq_pretrain_b200.benchmarks.tp_fused_1gpu [--only ag|rs|qk] [--iters 20] [--warmup 5]``

ncu does not run on multi-rank commands, so the one-kernel all-gather -> GEMM (``gather_gemm``)
and GEMM -> reduce-scatter (``gemm_scatter_reduce``, epilogue 5) are launched here exactly as
rank 0 launches them, with the peer's side prepared in this GPU's memory before the launch: the
peer's staged shard (all-gather) or its partial of rank 0's rows (reduce-scatter) sits in a local
buffer whose address stands in for the peer pointer, and the peer's publication flag / tile
stamps are set in advance. Nothing waits on another kernel: every flag the kernel polls is already
set, so each call is one self-contained launch. What differs from the real TP run: the peer rows
are read from local HBM instead of over NVLink, and no skew between ranks is absorbed. The shapes
are the fused-op sweep's at TP = 2 (column-parallel [8192/2, 2048] x [2048, 6144/2]; row-parallel
[8192, 6144/2] x [6144/2, 2048]); each result is checked against the plain GEMM.

Prints one JSON line per op: fused and plain-GEMM CUDA-event times (median after warm-up) and
the maximum relative error.
"""

from __future__ import annotations

import argparse
import json

import torch

HUGE = 1 << 60   # a flag value that every epoch of this run has reached


def _events(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return sorted(times)[len(times) // 2] if times else None


def _ptrs(*tensors):
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device="cuda")


def allgather_gemm(iters, warmup, rows=4096, k=2048, n=3072):
    from ..ops import _ext, gemm
    ops = _ext.ops()
    dev = torch.device("cuda")
    x_local = torch.randn(rows, k, device=dev, dtype=torch.bfloat16)
    w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
    peer_send = torch.randn(rows, k, device=dev, dtype=torch.bfloat16)    # rank 1's staged shard
    own_send = torch.empty(rows, k, device=dev, dtype=torch.bfloat16)
    flags = torch.zeros(2, 64, dtype=torch.int64, device=dev)             # [own area, rank 1's area]
    flags[0, 1] = HUGE                                                    # rank 1 published its shard
    chunk_flags = torch.zeros(2 * rows // 16, dtype=torch.int64, device=dev)
    own_done = torch.zeros(4, dtype=torch.int32, device=dev)
    peer_in, peer_ready = _ptrs(own_send, peer_send), _ptrs(flags[0], flags[1])
    xg = torch.empty(2 * rows, k, device=dev, dtype=torch.bfloat16)
    epoch = [0]

    def fused():
        epoch[0] += 1
        return ops.gather_gemm(xg, w, None, peer_in, flags[0].data_ptr(), chunk_flags, epoch[0], rows, 0, 2, False,
                               x_local=x_local, send_mine=own_send.data_ptr(), peer_ready=peer_ready,
                               own_done=own_done.data_ptr())

    y = fused()
    full = torch.cat((x_local, peer_send))
    ref = gemm.linear(full, w)
    err = float((y.float() - ref.float()).abs().max() / ref.float().abs().max())
    assert torch.equal(xg, full), "gathered rows differ"
    return dict(op="allgather_gemm (rank 0 of TP2, peer emulated locally)", shape=[2 * rows, k, n],
                fused_ms=_events(fused, iters, warmup), plain_gemm_ms=_events(lambda: gemm.linear(full, w), iters, warmup),
                max_rel_err=err, status=ops.gemm_status(True))


def gemm_reducescatter(iters, warmup, rows=4096, k=3072, n=2048):
    from ..ops import _ext, gemm
    ops = _ext.ops()
    dev = torch.device("cuda")
    x = torch.randn(2 * rows, k, device=dev, dtype=torch.bfloat16)
    w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
    own_recv = torch.zeros(2, rows, n, device=dev, dtype=torch.bfloat16)   # [source rank][rows][n]
    own_recv[1] = torch.randn(rows, n, device=dev, dtype=torch.bfloat16)    # rank 1's partial of our rows
    peer_recv = torch.zeros(2, rows, n, device=dev, dtype=torch.bfloat16)   # stands in for rank 1's slab
    tiles = (rows // 128) * -(-n // 256)
    slots = tiles * 8 * 4
    own_flags = torch.full((slots,), HUGE, dtype=torch.int64, device=dev)   # rank 1 stamped every tile
    peer_flags = torch.zeros(slots, dtype=torch.int64, device=dev)
    recv_ptrs, flag_ptrs = _ptrs(own_recv, peer_recv), _ptrs(own_flags, peer_flags)
    epoch = [0]

    def fused():
        epoch[0] += 1
        return ops.gemm_scatter_reduce(x, w, False, None, None, None, recv_ptrs, own_recv.data_ptr(), flag_ptrs,
                                       own_flags.data_ptr(), slots, epoch[0], rows, 0, 2)

    out = fused()
    full = gemm.linear(x, w).float()
    ref = full[:rows] + own_recv[1].float()
    err = float((out.float() - ref).abs().max() / ref.abs().max())
    sent = float((peer_recv[0].float() - full[rows:]).abs().max() / full[rows:].abs().max())
    return dict(op="gemm_reducescatter (rank 0 of TP2, peer emulated locally)", shape=[2 * rows, k, n],
                fused_ms=_events(fused, iters, warmup), plain_gemm_ms=_events(lambda: gemm.linear(x, w), iters, warmup),
                max_rel_err=max(err, sent), status=ops.gemm_status(True))


def qk_norm_rope(iters, warmup, rows=32768, width=768, hd=128):
    """Wan q / k full-width RMSNorm + RoPE (one kernel each way) at the T2V workload's per-rank TP2 shape,
    with the row-sum exchange running against this GPU's own slabs (tp = 1: the publish / flag /
    acquire steps execute, the peer is this rank)."""
    from ..ops import _ext
    ops = _ext.ops()
    dev = torch.device("cuda")
    max_rows = 2 * rows
    flags = torch.zeros(-(-max_rows // 64) * 8, dtype=torch.int64, device=dev)
    slabs = [torch.zeros(max_rows, dtype=torch.float32, device=dev) for _ in range(2)]
    ctr = torch.zeros(1, dtype=torch.int64, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    kw = dict(peer_recv=_ptrs(slabs[0]), my_recv=slabs[0].data_ptr(), peer_flags=_ptrs(flags),
              my_flags=flags.data_ptr(), rank=0, tp=1, max_rows=max_rows, epoch_ctr=ctr.data_ptr(),
              epoch_done=done.data_ptr(), peer_recv_odd=_ptrs(slabs[1]), my_recv_odd=slabs[1].data_ptr())
    q = torch.randn(rows, width, device=dev, dtype=torch.bfloat16)
    kv = torch.randn(rows, 2 * width, device=dev, dtype=torch.bfloat16)
    k = kv[:, :width]                                   # the kv projection's k half, row-strided
    wq, wk = torch.rand(width, device=dev) + 0.5, torch.rand(width, device=dev) + 0.5
    ang = torch.rand(rows, hd // 2, device=dev) * 6.28
    cos, sin = ang.cos(), ang.sin()
    fwd = lambda: ops.qk_norm_rope_fwd(q, k, wq, wk, cos=cos, sin=sin, head_dim=hd, total_dim=2 * width, eps=1e-6,
                                       **kw)
    yq, yk, rstd = fwd()
    dyq, dyk = torch.randn_like(yq), torch.randn_like(yk)
    bwd = lambda: ops.qk_norm_rope_bwd(dyq, dyk, q, k, wq, wk, rstd, cos=cos, sin=sin, head_dim=hd,
                                       total_dim=2 * width, **kw)
    t_f, t_b = _events(fwd, iters, warmup), _events(bwd, iters, warmup)
    tensor = rows * width * 2
    angles = 2 * rows * (hd // 2) * 4
    f_bytes, b_bytes = 4 * tensor + angles, 6 * tensor + angles   # fwd: q, k in / out; bwd: dy, x in, dx out
    return dict(op="wan q/k rmsnorm + rope (exchange against own slabs)", shape=[rows, width, hd],
                fwd_ms=t_f, bwd_ms=t_b, fwd_gbs=f_bytes / t_f / 1e6, bwd_gbs=b_bytes / t_b / 1e6,
                comm_status=ops.comm_status_read(True))


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--only", choices=("ag", "rs", "qk"), default=None)
    parser.add_argument("--iters", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    args = parser.parse_args()
    torch.manual_seed(0)
    if args.only in (None, "ag"):
        print(json.dumps(allgather_gemm(args.iters, args.warmup)), flush=True)
    if args.only in (None, "rs"):
        print(json.dumps(gemm_reducescatter(args.iters, args.warmup)), flush=True)
    if args.only in (None, "qk"):
        print(json.dumps(qk_norm_rope(args.iters, args.warmup)), flush=True)


if __name__ == "__main__":
    main()
