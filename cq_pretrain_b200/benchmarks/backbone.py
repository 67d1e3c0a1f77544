"""Backbone step benchmark: forward / backward / optimizer time of the CQ model, max over ranks.

``[torchrun --nproc-per-node N] python -m cq_pretrain_b200.benchmarks.backbone [--mode i2t|joint]
[--lengths 2048 8192] [--steps 5] [--warmup 3]`` builds the Qwen3.5-2B CQ backbone (``joint``
adds the Wan2.1-1.3B renderer and T2I targets) with random weights, packs synthetic documents
with resident N(0,1) merger features and latents, and times each phase with CUDA events
(reference ``scripts/benchmark_backbones.py:26-227``; the Gemma comparison model of the
reference is not part of this framework). TP = 2 when N >= 2. One JSON line per length.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--mode", choices=("i2t", "joint"), default="joint")
    parser.add_argument("--lengths", type=int, nargs="+", default=[2048, 8192])
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--tp", type=int, default=None)
    args = parser.parse_args()
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist
    from ..config import qwen35_2b_wan
    from ..data.synthetic import synthetic_batch
    from ..parallel import state as ps
    from ..train.loss import compose_losses
    from ..train.trainer import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp = args.tp or (2 if world >= 2 else 1)
    st = ps.initialize(tp, timeout_s=600.0)
    cfg = qwen35_2b_wan(visual_query_mode="fixed", image_condition_queries=256)
    trainer = Trainer(cfg, tp=tp, lr=5e-5, ema_decay=0.999 if args.mode == "joint" else None)
    for length in args.lengths:
        host, receipt = synthetic_batch(cfg, length, seed=7 + st.dp_rank, kind="joint", images=2, grid=(1, 64, 64),
                                        latent_shape=(16, 1, 64, 64), understanding="all" if args.mode == "i2t" else False,
                                        pad_multiple=128 * tp)
        batch = trainer.preparer(host.pin_memory(), receipt, non_blocking=True)
        phases = {"forward": [], "backward": [], "optimizer": []}
        for step in range(args.warmup + args.steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            trainer.optimizer.zero_grad()
            ev[0].record()
            out = trainer.model(batch)
            losses = compose_losses(out, cfg, (1.0, 1.0))
            ev[1].record()
            losses["loss"].backward()
            ev[2].record()
            trainer.optimizer.finish_grad_sync()
            trainer.optimizer.step(5e-5)
            ev[3].record()
            torch.cuda.synchronize()
            if step >= args.warmup:
                for k, (a, b) in zip(phases, ((0, 1), (1, 2), (2, 3))):
                    phases[k].append(ev[a].elapsed_time(ev[b]))
        med = torch.tensor([statistics.median(v) for v in phases.values()], dtype=torch.float64,
                           device=trainer.device)
        if world > 1:
            dist.all_reduce(med, op=dist.ReduceOp.MAX)
        fwd, bwd, opt = med.tolist()
        step_ms = fwd + bwd + opt
        if st.rank == 0:
            print(json.dumps(dict(mode=args.mode, content_tokens=length, tp=tp, dp=st.dp, forward_ms=round(fwd, 3),
                                  backward_ms=round(bwd, 3), optimizer_ms=round(opt, 3), step_ms=round(step_ms, 3),
                                  content_tokens_per_s=round(length * st.dp / step_ms * 1000, 1),
                                  peak_gib=round(torch.cuda.max_memory_allocated() / 2 ** 30, 2))), flush=True)
    if world > 1:
        dist.barrier()
        ps.destroy()


if __name__ == "__main__":
    main()
