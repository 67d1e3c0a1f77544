"""Joint T2V + V2T training step (Qwen3.5-2B + Wan2.1-1.3B, bf16).

``[torchrun --nproc-per-node N] python -m cq_pretrain_b200.benchmarks.t2v [--tp T] [--steps K]``
packs one T2V document (81 frames at 480x832: a 16x21x60x104 latent = 32,760 DiT tokens; Qwen
content of 8 frames = 1,560 merged tokens and, with native visual queries, 1,560 queries), one
V2T document of the same geometry and 4,096 tokens of text documents into one 8K pack per DP
rank, then times full training steps (forward, the chunked DiT backward, the backbone backward,
gradient reduction, AdamW + EMA): CUDA events per step after warm-up, the max over ranks. Synthetic
data and random-init weights. ``--checkpoint-dit`` recomputes the DiT blocks in backward (the
activation budget of one 32K-token target), ``--recompute`` the backbone layers.
Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import time


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--tp", type=int, default=None, help="TP size (default: the world size, at most 4)")
    parser.add_argument("--steps", type=int, default=4)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--length", type=int, default=8192)
    parser.add_argument("--checkpoint-dit", type=int, default=0, help="recompute this many DiT blocks (30 = all)")
    parser.add_argument("--recompute", type=int, default=0)
    args = parser.parse_args()
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from ..config import qwen35_2b_wan
    from ..data.synthetic import synthetic_batch
    from ..parallel import state as ps
    from ..train.trainer import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp = args.tp or min(world, 4)
    st = ps.initialize(tp, timeout_s=900.0)
    cfg = qwen35_2b_wan(visual_query_mode="native", checkpoint_backbone=args.recompute,
                        checkpoint_dit_layers=args.checkpoint_dit)
    cfg.validate(tp)
    host, receipt = synthetic_batch(cfg, args.length, seed=7 + st.dp_rank, kind="video", pad_multiple=128 * tp)
    host = host.pin_memory()
    trainer = Trainer(cfg, tp=tp, lr=5e-5, ema_decay=0.999)
    for _ in range(args.warmup):
        trainer.train_step([(host, receipt)])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.reset_peak_memory_stats()
    ms, wall0 = [], time.perf_counter()
    for _ in range(args.steps):
        ms.append(trainer.train_step([(host, receipt)], timing=True)["compute_ms"])
    torch.cuda.synchronize()
    wall = (time.perf_counter() - wall0) * 1000 / args.steps
    stats = torch.tensor([sum(ms) / len(ms), wall, torch.cuda.max_memory_allocated() / 2 ** 30],
                         dtype=torch.float64, device=trainer.device)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    step_ms, wall_ms, peak = stats.tolist()
    gen = host.generation
    if st.rank == 0:
        print(json.dumps(dict(
            config="joint T2V + V2T, Qwen3.5-2B + Wan2.1-1.3B", n_gpus=world,
            parallelism=f"tp{tp}xdp{st.dp}", ms_per_step=round(step_ms, 2), wall_ms_per_step=round(wall_ms, 2),
            content_tokens_per_s=round(args.length * st.dp / (step_ms / 1000), 1),
            dit_tokens_per_step=int(sum(gen.lengths)) * st.dp,
            dit_tokens_per_s=round(sum(gen.lengths) * st.dp / (step_ms / 1000), 1),
            rows=int(host.mainline.rows), queries=int(host.mainline.queries),
            text_targets=int(host.text_indices.numel()), peak_gib=round(peak, 1),
            checkpoint_dit_layers=args.checkpoint_dit, recompute_backbone=args.recompute,
            steps=args.steps, warmup=args.warmup, data="synthetic (random-init weights)")), flush=True)
    trainer.close()
    if world > 1:
        ps.destroy()


if __name__ == "__main__":
    main()
