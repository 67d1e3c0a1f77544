"""Per-kernel device-time breakdown of one joint training step (torch.profiler, CUPTI).

``[torchrun --nproc-per-node N] python -m cq_pretrain_b200.benchmarks.profile_step [--length 8192]
[--recompute 1] [--tp T]`` runs the bench configuration (TP = T, default N; DP = N / T; rank 0
reports), warms up, profiles one step and prints the kernels with the largest total device time,
grouped by name, plus each group's share of the step, and where the device sat idle: the step's
span on the device timeline against the union of its kernels, the idle time inside each phase
(backbone forward / backward, renderer forward / backward, optimizer, from the phase timer's profiler ranges), and
the kernels that most often waited for their launch (idle gap before them > 2 us), which marks the
host-bound stretches.
"""

from __future__ import annotations

import argparse
import json

import torch


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--length", type=int, default=8192)
    parser.add_argument("--recompute", type=int, default=1)
    parser.add_argument("--top", type=int, default=40)
    parser.add_argument("--layers", type=int, default=None)
    parser.add_argument("--tp", type=int, default=None, help="TP size under torchrun (default: the world size)")
    parser.add_argument("--images", type=int, default=3)
    args = parser.parse_args()
    import os

    from ..config import qwen35_2b_wan
    from ..data.synthetic import synthetic_batch
    from ..parallel import state as ps
    from ..train.trainer import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp = args.tp or world
    st = ps.initialize(tp, timeout_s=600.0) if world > 1 else None   # DP = world / TP

    cfg = qwen35_2b_wan(visual_query_mode="fixed", image_condition_queries=256, checkpoint_backbone=bool(args.recompute))
    if args.layers:
        cfg.layers = args.layers
    seed = 42 + (st.dp_rank if st is not None else 0)
    host, receipt = synthetic_batch(cfg, args.length, seed=seed, kind="joint", images=args.images, grid=(1, 64, 64),
                                    latent_shape=(16, 1, 64, 64), understanding=True, pad_multiple=128 * tp)
    host = host.pin_memory()
    trainer = Trainer(cfg, tp=tp, lr=5e-5, ema_decay=0.999)
    for _ in range(3):
        trainer.train_step([(host, receipt)])
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile

    from ..utils.observe import PhaseTimer
    timer = PhaseTimer(trainer.device, annotate=True)
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
        trainer.train_step([(host, receipt)], phases=timer)
        torch.cuda.synchronize()
    trainer.close()
    if st is not None and st.rank != 0:
        ps.destroy()
        return
    events = prof.key_averages()
    phase_names = {"forward", "backward", "renderer_forward", "renderer_backward", "optimizer"}
    kernels = [e for e in events if e.device_type.name == "CUDA" and e.key not in phase_names]
    total = sum(e.self_device_time_total for e in kernels)
    rows = sorted(kernels, key=lambda e: -e.self_device_time_total)[: args.top]
    print(json.dumps(dict(total_device_ms=round(total / 1000, 2), peak_gib=round(torch.cuda.max_memory_allocated() / 2**30, 1))))
    print("== kernels ==")
    for e in rows:
        print(f"{e.self_device_time_total / 1000:9.2f} ms {100 * e.self_device_time_total / total:5.1f}% {e.count:6d}x  {e.key[:110]}")
    print("== aten ops by input shape (device time of their kernels) ==")
    shaped = [e for e in prof.key_averages(group_by_input_shape=True)
              if e.key.startswith("aten::") and e.device_type.name == "CPU"]
    for e in sorted(shaped, key=lambda e: -e.device_time_total)[: args.top]:
        print(f"{e.device_time_total / 1000:9.2f} ms {e.count:6d}x  {e.key:28s} {str(e.input_shapes)[:120]}")
    idle_report(prof, args.top)
    if st is not None:
        ps.destroy()


def idle_report(prof, top):
    """Device-timeline gaps of the profiled step, by phase range and by the kernel after each gap."""
    spans, ranges = [], []
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        (ranges if getattr(e, "is_user_annotation", False) else spans).append(
            (e.time_range.start, e.time_range.end, e.name))
    if not spans:
        return
    spans.sort()
    busy, gaps, end, last = 0.0, [], spans[0][0], ""
    for a, b, name in spans:
        if a > end:
            gaps.append((end, a, name, last))
        busy += max(0.0, b - max(a, end))
        if b >= end:
            end, last = b, name
    span = end - spans[0][0]
    print(json.dumps(dict(device_span_ms=round(span / 1000, 2), kernel_union_ms=round(busy / 1000, 2),
                          idle_ms=round((span - busy) / 1000, 2), gaps=len(gaps))))
    phases = [(a, b, n) for a, b, n in ranges if n in ("forward", "backward", "renderer_forward", "renderer_backward",
                                                     "optimizer")]
    by_phase: dict = {}
    def label_of(a, b):
        mid = (a + b) / 2
        inside = [(t - s, n) for s, t, n in phases if s <= mid < t]
        return min(inside)[1] if inside else "between phases"

    for a, b, _, _ in gaps:
        label = label_of(a, b)
        by_phase[label] = by_phase.get(label, 0.0) + (b - a)
    print("== idle by phase ==")
    for label, us in sorted(by_phase.items(), key=lambda kv: -kv[1]):
        print(f"{us / 1000:9.2f} ms  {label}")
    waited: dict = {}
    print("== largest gaps ==")
    t0 = spans[0][0]
    for a, b, name, prev in sorted(gaps, key=lambda g: g[0] - g[1])[:12]:
        print(f"{(b - a) / 1000:9.2f} ms at {(a - t0) / 1000:8.2f} ms  [{label_of(a, b)}]  {prev[:50]} -> {name[:50]}")
    for a, b, name, _ in gaps:
        if b - a > 2.0:
            n, t = waited.get(name, (0, 0.0))
            waited[name] = (n + 1, t + (b - a))
    print("== kernels launched after an idle gap (> 2 us) ==")
    for name, (n, us) in sorted(waited.items(), key=lambda kv: -kv[1][1])[:top]:
        print(f"{us / 1000:9.2f} ms {n:6d}x  {name[:110]}")


if __name__ == "__main__":
    main()
