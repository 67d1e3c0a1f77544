"""LM-head + cross-entropy benchmark (8192 tokens x 2048 x 248K vocab).

``[torchrun --nproc-per-node N] python -m cq_pretrain_b200.benchmarks.ce [--rows 8192] [--chunk 1024]``
times forward+backward of ``ops.cross_entropy.linear_cross_entropy`` (GEMM epilogues that fold
the logits into online softmax statistics and write softmax gradients, vocabulary split over TP
ranks; under TP the statistics cross NVLink inside one kernel unless ``--no-fused``) against the same loss through materialised fp32 logits and ``F.cross_entropy``
(single GPU only). CUDA events, median of ``--iters`` after 3 warm-ups, max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--rows", type=int, default=8192)
    parser.add_argument("--hidden", type=int, default=2048)
    parser.add_argument("--vocab", type=int, default=248320)
    parser.add_argument("--chunk", type=int, default=1024)
    parser.add_argument("--iters", type=int, default=10)
    parser.add_argument("--no-reference", action="store_true")
    parser.add_argument("--no-fused", action="store_true", help="TP: NCCL all-reduces instead of the in-kernel exchange")
    args = parser.parse_args()
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    from ..ops.cross_entropy import linear_cross_entropy
    from ..parallel import state as ps

    world = int(os.environ.get("WORLD_SIZE", "1"))
    st = ps.initialize(world, timeout_s=300.0)
    if world > 1 and not args.no_fused:
        from ..parallel import symmetric
        symmetric.enable()
    torch.manual_seed(0)
    dev = st.device
    h = (torch.randn(args.rows, args.hidden, device=dev) * 0.5).to(torch.bfloat16).requires_grad_()
    shard = args.vocab // st.tp
    w = (torch.randn(shard, args.hidden, device=dev) * 0.02).to(torch.bfloat16).requires_grad_()
    t = torch.randint(0, args.vocab, (args.rows,), device=dev)

    def fused():
        h.grad = w.grad = None
        linear_cross_entropy(h, w, t, args.chunk).backward()

    def reference():
        h.grad = w.grad = None
        F.cross_entropy((h @ w.T).float(), t).backward()

    def timed(fn):
        for _ in range(3):
            fn()
        times = []
        for _ in range(args.iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        v = torch.tensor([statistics.median(times)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return v.item()

    row = dict(rows=args.rows, hidden=args.hidden, vocab=args.vocab, tp=st.tp, fused_ms=round(timed(fused), 3),
               stats_exchange="nccl" if world == 1 or args.no_fused else "in-kernel")
    flops = 6.0 * args.rows * args.hidden * args.vocab / st.tp   # logits fwd + dh + dW
    row["fused_tflops"] = round(flops / row["fused_ms"] / 1e9, 1)
    if world == 1 and not args.no_reference:
        row["reference_ms"] = round(timed(reference), 3)
    if st.rank == 0:
        print(json.dumps(row), flush=True)
    if world > 1:
        dist.barrier()
        if not args.no_fused:
            from ..parallel import symmetric
            row_status = symmetric.status()
            assert row_status == dict(gemm=0, comm=0), row_status
            symmetric.disable()
        ps.destroy()


if __name__ == "__main__":
    main()
