"""Flagship benchmark: joint T2I+I2T training step, Qwen3.5-2B + Wan2.1-1.3B, 8K packed tokens.

``python bench.py --gpus N --steps K --warmup W`` (N > 1 under ``torch.distributed.run``). Each
DP rank trains on one synthetic 8192-token pack per step (random-init weights, synthetic
merger features and latents of the production-model shape). The pack is a joint T2I + I2T pack:
two T2I documents (caption -> 512x512 image: 1024 merger tokens, 256 visual queries and a
16x1x64x64 Wan target each), one I2T document (image -> caption) and log-uniform text documents
filling the rest. TP is 2 from N = 2 up (TP2 x DP N/2; the headline target is TP2 x DP4 on 8
GPUs) and 1 on a single GPU.

Reported: ``value`` = content tokens/s of the whole job, from CUDA-event device time of the
compute of K steps (max over ranks); ``e2e`` = the same metric from host wall time of K calls of
the public ``Trainer.train_step`` API, each including the pinned host->device copy of the pack
and the device->host read of the loss. Working set per step (weights, optimizer state) is
far larger than the 126 MB L2, so no explicit flush is needed between iterations.
``--impl reference`` reports why the reference cannot run here.

Extra keys: ``gdn_fwd_bwd_ms`` (the GDN layer microbenchmark: one layer forward+backward at 2048 and
8192 content tokens with 32 and 16 value heads, median of 12 after 3 warm-ups, heads split over
TP when N > 1) and, for N > 1, ``fused_tp_check``: the maximum relative error of every in-kernel
TP collective against NCCL on the live process group, run once before the warm-up.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

METRIC = "joint train step s & tokens/s at 8K (box, max over ranks) 1/2/4/8 B200; GDN fwd+bwd ms"
BASELINE_TOKENS_PER_GPU = 8 * 8192 / 1.946 / 16  # reference: 1.946 s joint 8K step, 16x 910B, TP2xDP8, batch 8


def reference_unavailable(args):
    reason = ("reference needs torch_npu + HCCL + AscendC kernels (training/train.py:240, "
              "distributed/megatron.py:64, ops/gated_delta_net.py:24-57); its only non-NPU GDN path is the "
              "per-token recurrent oracle (models/backbone_qwen35.py:56-73) whose autograd graph at the 8K "
              "config needs ~300 GB")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason, "n_gpus": args.gpus}), flush=True)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path, gpus):
        self.path, self.gpus, self.proc = path, gpus, None

    def start(self):
        try:
            self.handle = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.handle, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"])
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.handle.close()
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        indices = [int(x) for x in visible.split(",")] if visible else list(range(self.gpus))
        indices = set(indices[: self.gpus])
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in indices:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(mx) if mx else None,
                    reasons=sorted(reasons), samples=len(sm))


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="ours", choices=("ours", "reference"))
    parser.add_argument("--tp", type=int, default=None)
    parser.add_argument("--length", type=int, default=8192)
    parser.add_argument("--images", type=int, default=3, help="visual documents per pack (all but one are T2I)")
    parser.add_argument("--no-gdn", action="store_true", help="skip the GDN layer microbenchmark timings")
    parser.add_argument("--clocks-csv", default=None, help="where to keep the nvidia-smi samples (default: a temp file)")
    parser.add_argument("--layers", type=int, default=None, help="debug only: fewer layers (invalid as a bench value)")
    parser.add_argument("--recompute", type=int, default=0, help="recompute backbone layers in backward")
    args = parser.parse_args()
    if args.impl == "reference":
        reference_unavailable(args)
        return
    if args.warmup < 3:
        raise SystemExit("at least 3 warm-up steps are required")

    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist
    from cq_pretrain_b200.config import qwen35_2b_wan
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.ops import _ext
    from cq_pretrain_b200.parallel import state as ps
    from cq_pretrain_b200.train.trainer import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    tp = args.tp or (2 if args.gpus >= 2 else 1)
    st = ps.initialize(tp, timeout_s=600.0)
    rank = st.rank
    cfg = qwen35_2b_wan(visual_query_mode="fixed", image_condition_queries=256,
                        checkpoint_backbone=args.recompute)
    if args.layers:
        cfg.layers, cfg.dit_layers = args.layers, max(1, args.layers)
    cfg.validate(tp)
    grid, latent = (1, 64, 64), (16, 1, 64, 64)
    host, receipt = synthetic_batch(cfg, args.length, seed=42 + st.dp_rank, kind="joint", images=args.images,
                                    grid=grid, latent_shape=latent, understanding=True, pad_multiple=128 * tp)
    host = host.pin_memory()
    trainer = Trainer(cfg, tp=tp, lr=5e-5, ema_decay=0.999)
    h2d = sum(t.numel() * t.element_size() for t in _tensors(host))
    check = None
    if world > 1:
        from cq_pretrain_b200.parallel.selfcheck import fused_vs_nccl
        check = fused_vs_nccl()
    for _ in range(args.warmup):
        trainer.train_step([(host, receipt)])
    torch.cuda.synchronize()
    clocks_path = args.clocks_csv or os.path.join(tempfile.gettempdir(), f"cqb_clocks_n{args.gpus}_{os.getpid()}.csv")
    sampler = ClockSampler(clocks_path, args.gpus) if st.tp_rank == 0 and st.dp_rank == 0 else None
    if sampler:
        sampler.start()
    launches0 = _ext.launches()
    compute_ms = 0.0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for _ in range(args.steps):
        metrics = trainer.train_step([(host, receipt)], timing=True)
        compute_ms += metrics["compute_ms"]
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    launches = _ext.launches() - launches0
    clocks = sampler.stop() if sampler else None
    timing = torch.tensor([compute_ms, wall * 1000.0], dtype=torch.float64, device=trainer.device)
    if world > 1:
        dist.all_reduce(timing, op=dist.ReduceOp.MAX)
    compute_ms, wall_ms = timing.tolist()
    tokens_per_step = args.length * st.dp
    ms_per_step = compute_ms / args.steps
    pack = _composition(host)
    trainer.close()   # captured graphs (which may hold NCCL work) go before the process group
    del trainer
    torch.cuda.empty_cache()
    gdn = None
    if not args.no_gdn and not args.layers:
        from cq_pretrain_b200.benchmarks import gdn as gdn_bench
        gdn = {f"{r['content_tokens']}_v{r['value_heads']}": r["median_ms"]
               for heads in (32, 16) for r in gdn_bench.measure([2048, 8192], heads)}
        gdn["tp"] = tp
        gdn["reference_910b_ms"] = {"2048": 10.46, "8192": 38.60}
    value = tokens_per_step / (ms_per_step / 1000.0)
    e2e = tokens_per_step / (wall_ms / args.steps / 1000.0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "content tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / (BASELINE_TOKENS_PER_GPU * args.gpus), 3),
            "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) merger features and latents)",
            "config": {"model": "Qwen3.5-2B-hybrid(24L: 18 GDN + 6 gated-attn) + Wan2.1-T2V-1.3B",
                       "global_batch": st.dp, "seq_len": args.length, "parallelism": f"tp{tp}xdp{st.dp}",
                       "pack": pack, "images_per_pack": args.images, "merger_tokens_per_image": 1024,
                       "visual_queries_per_image": 256, "latent": "16x1x64x64",
                       "rows_per_pack": int(host.mainline.rows), "gdn_events": host.mainline.delta.events,
                       "l2": "working set (weights + optimizer state) >> 126 MB L2; no flush",
                       "layers_override": args.layers, "recompute_backbone": bool(args.recompute)},
            "e2e": {"value": round(e2e, 1), "unit": "content tokens/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": 16},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "loss": metrics["loss"],
            "gdn_fwd_bwd_ms": gdn,
            "fused_tp_check": check,
            "baseline": {"tokens_per_s_per_gpu": round(BASELINE_TOKENS_PER_GPU, 1),
                         "source": "reference 1.946 s joint 8K step on 16x 910B TP2xDP8, global batch 8"},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        ps.destroy()


def _composition(batch):
    """Document mix of one pack: T2I targets, I2T images, text documents, rows and queries."""
    gen = batch.generation
    targets = int(batch.generation_image_count)
    images = int(batch.image_indices.shape[0])
    return dict(t2i_targets=targets, i2t_images=images - targets,
                dit_tokens=int(sum(gen.lengths)) if gen is not None else 0,
                rows=int(batch.mainline.rows), queries=int(batch.mainline.queries),
                text_targets=int(batch.text_indices.numel()))


def _tensors(batch):
    import torch
    out = []

    def walk(x):
        if isinstance(x, torch.Tensor):
            out.append(x)
        elif hasattr(x, "__dataclass_fields__"):
            for f in x.__dataclass_fields__:
                walk(getattr(x, f))
        elif isinstance(x, tuple):
            for y in x:
                walk(y)

    walk(batch)
    return out


if __name__ == "__main__":
    main()
