"""GEMM microbenchmark: the tcgen05 kernels vs cuBLAS (torch.matmul) on the model's shapes.

``python -m cq_pretrain_b200.benchmarks.gemm [--shapes M,N,K ...] [--only fwd|dgrad|wgrad]``
prints one JSON line per shape with CUDA-event times (median of 20 after 5 warm-ups) and
TFLOP/s for: forward ``x W^T``, input gradient ``dY W`` and fp32 weight-gradient accumulation,
next to cuBLAS (``torch.matmul``) on the same operands. ``--iters 1 --warmup 1`` gives the
small single-launch case used for ncu captures.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch

from ..ops import _ext

SHAPES = [  # (rows, out, in): Qwen3.5-2B at 16K CQ rows, Wan at 2K tokens
    (16384, 8224, 2048), (16384, 2048, 2048), (16384, 12288, 2048), (16384, 2048, 6144),
    (16384, 4096, 2048), (2048, 8960, 1536), (2048, 1536, 8960), (8192, 8192, 8192),
]


def timed(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times)


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--shapes", nargs="+", default=None, help="M,N,K triples")
    parser.add_argument("--only", choices=("fwd", "dgrad", "wgrad"), default=None)
    parser.add_argument("--iters", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--no-cublas", action="store_true")
    args = parser.parse_args()
    shapes = [tuple(int(v) for v in s.split(",")) for s in args.shapes] if args.shapes else SHAPES
    ops = _ext.ops()
    kinds = [args.only] if args.only else ["fwd", "dgrad", "wgrad"]
    for m, n, k in shapes:
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
        dy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
        acc = torch.zeros(n, k, device="cuda", dtype=torch.float32)
        flops = 2.0 * m * n * k
        row = dict(m=m, n=n, k=k)
        ours = dict(fwd=lambda: ops.gemm_nt(x, w, None), dgrad=lambda: ops.gemm_nn(dy, w),
                    wgrad=lambda: ops.gemm_tn_acc(dy, x, acc))
        cublas = dict(fwd=lambda: x @ w.T, dgrad=lambda: dy @ w,
                      wgrad=lambda: acc.add_(torch.mm(dy.T, x, out_dtype=torch.float32)))
        for kind in kinds:
            row[f"{kind}_ours_ms"] = timed(ours[kind], args.iters, args.warmup)
            if not args.no_cublas:
                row[f"{kind}_cublas_ms"] = timed(cublas[kind], args.iters, args.warmup)
        for key in list(row):
            if key.endswith("_ms"):
                row[key.replace("_ms", "_tflops")] = round(flops / row[key] / 1e9, 1)
        assert ops.gemm_status(True) == 0
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
