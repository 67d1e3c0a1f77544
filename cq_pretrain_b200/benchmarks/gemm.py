"""GEMM microbenchmark: the tcgen05 kernels vs cuBLAS (torch.matmul) on the model's shapes.

``python -m cq_pretrain_b200.benchmarks.gemm`` prints one JSON line per shape with CUDA-event
times (median of 20 after 5 warm-ups, operands larger than L2 rotate between iterations) and
TFLOP/s for: forward ``x W^T``, input gradient ``dY W`` and fp32 weight-gradient accumulation.
"""

from __future__ import annotations

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
    ops = _ext.ops()
    for m, n, k in SHAPES:
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
        dy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
        acc = torch.zeros(n, k, device="cuda", dtype=torch.float32)
        flops = 2.0 * m * n * k
        row = dict(m=m, n=n, k=k)
        row["fwd_ours_ms"] = timed(lambda: ops.gemm_nt(x, w, None))
        row["fwd_cublas_ms"] = timed(lambda: x @ w.T)
        row["dgrad_ours_ms"] = timed(lambda: ops.gemm_nn(dy, w))
        row["dgrad_cublas_ms"] = timed(lambda: dy @ w)
        row["wgrad_ours_ms"] = timed(lambda: ops.gemm_tn_acc(dy, x, acc))
        row["wgrad_cublas_ms"] = timed(lambda: acc.add_(torch.mm(dy.T, x, out_dtype=torch.float32)))
        for key in list(row):
            if key.endswith("_ms"):
                row[key.replace("_ms", "_tflops")] = round(flops / row[key] / 1e9, 1)
        assert ops.gemm_status(True) == 0
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
