"""Gated-DeltaNet layer forward+backward microbenchmark.

``python -m cq_pretrain_b200.benchmarks.gdn [--lengths 2048 8192] [--value-heads 32 16] [--iterations 12]``
builds one GDN layer of the Qwen3.5-2B shape with 16 q/k heads and 32 (the microbenchmark's) or 16 (the
reference's published run) v heads of dim 128 (short conv 4,
gated RMSNorm output), random N(0, 0.02) weights, and the CQ event plan of a synthetic pack
(2 T2I images, text documents with a boundary every 1024 tokens). Each iteration runs the
layer forward and backward on N(0, 1) bf16 activations; 3 warm-ups, then the median of the
CUDA-event times (reference ``scripts/benchmark_gdn.py:16-67``). Under ``torchrun`` with 2
ranks the heads are split over TP=2 and the time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics


def build_layer(value_heads, device):
    """One GDN layer of the Qwen3.5-2B shape (16 q/k heads x 128) with ``value_heads`` value heads,
    N(0, 0.02) matrix weights, bf16 except the fp32 ``A_log`` and gated-norm weight."""
    import torch
    from ..config import qwen35_2b_wan
    from ..models.qwen35 import GatedDelta

    torch.manual_seed(872)
    cfg = qwen35_2b_wan(linear_value_heads=value_heads)
    layer = GatedDelta(cfg).to(device)
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if p.dim() >= 2:
                p.normal_(0.0, 0.02)
    layer = layer.to(torch.bfloat16)
    layer.A_log.data = layer.A_log.data.float()
    layer.norm.weight.data = layer.norm.weight.data.float()
    return cfg, layer


def measure(lengths, value_heads=32, iterations=12, warmup=3, profile=False):
    """Median CUDA-event ms of one layer forward+backward per content length (max over ranks; under
    TP the heads are split over the TP group). Returns one dict per length."""
    import torch
    import torch.distributed as dist
    from ..data.synthetic import synthetic_batch
    from ..parallel import state as ps

    st = ps.state()
    world = dist.get_world_size() if dist.is_initialized() else 1
    cfg, layer = build_layer(value_heads, st.device)
    rows_out = []
    for length in lengths:
        host, _ = synthetic_batch(cfg, length, seed=0, kind="gdn", pad_multiple=128 * st.tp)
        batch = host.to(st.device)
        plan = batch.mainline
        gen = torch.Generator(device=st.device).manual_seed(1 + st.rank)
        x = torch.randn(plan.rows // st.tp, cfg.width, device=st.device, generator=gen).to(torch.bfloat16)
        x.requires_grad_(True)
        upstream = torch.randn(x.shape, device=st.device, generator=gen).to(torch.bfloat16) / 100

        def step():
            layer.zero_grad(set_to_none=True)
            x.grad = None
            y = layer(x, plan)
            (y.float() * upstream.float()).sum().backward()
            return y

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        times = []
        for _ in range(iterations):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            start.record()
            step()
            end.record()
            torch.cuda.synchronize()
            times.append(start.elapsed_time(end))
        t = torch.tensor(times, dtype=torch.float64, device=st.device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times = t.tolist()
        row = dict(content_tokens=length, value_heads=value_heads, tp=st.tp, query_tokens=int(plan.queries),
                   events=int(plan.delta.events), rows=int(plan.rows), median_ms=round(statistics.median(times), 3),
                   samples_ms=[round(v, 3) for v in times], peak_bytes=int(torch.cuda.max_memory_allocated()),
                   reference_910b_ms={2048: 10.46, 8192: 38.60}.get(length))
        rows_out.append(row)
        if profile and st.rank == 0:
            from torch.profiler import ProfilerActivity, profile as prof_ctx
            with prof_ctx(activities=[ProfilerActivity.CUDA]) as prof:
                step()
                torch.cuda.synchronize()
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=25, max_name_column_width=90),
                  flush=True)
    return rows_out


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--lengths", type=int, nargs="+", default=[2048, 8192])
    parser.add_argument("--value-heads", type=int, nargs="+", default=[32, 16])
    parser.add_argument("--iterations", type=int, default=12)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--output", default=None)
    parser.add_argument("--profile", action="store_true", help="also print the top kernels of one iteration")
    args = parser.parse_args()
    import torch
    import torch.distributed as dist
    from ..parallel import state as ps

    world = int(os.environ.get("WORLD_SIZE", "1"))
    st = ps.initialize(world, timeout_s=300.0)
    report = dict(device=torch.cuda.get_device_name(0), tp=st.tp, results=[])
    for heads in args.value_heads:
        for row in measure(args.lengths, heads, args.iterations, args.warmup, args.profile):
            report["results"].append(row)
            if st.rank == 0:
                print(json.dumps(row), flush=True)
    if st.rank == 0 and args.output:
        with open(args.output, "w") as f:
            json.dump(report, f, indent=2)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
