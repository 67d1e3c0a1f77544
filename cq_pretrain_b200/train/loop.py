"""The training program (``python -m cq_pretrain_b200.train.loop``), one process per GPU.

Reference ``training/train.py:160-871``. Per update: read ``grad_accum`` packs per DP rank from
the consumed-only loader (a DP all-reduce of counts ends training when every rank is
exhausted), run ``Trainer.train_step``, then acknowledge the packs (the resumable cursor only
moves after a committed update), write ``steps.jsonl`` (step time = max over ranks, content
tokens/s, peak memory, losses, grad norm, lr), and checkpoint / snapshot / prune on interval.
Startup writes ``run.json`` (versions, topology, parameter counts, source digest); shutdown
writes ``summary.json`` (mean / median / p95 over post-warm-up steps) and, per rank,
``backend_rank_XXXXX.json`` (native library path and sha256, devices, versions, launch counts).
Every rank appends ``timing_rank_XXXXX.jsonl`` (step seconds, data-wait seconds, and with
``--phase-timing`` forward / backward / optimizer milliseconds) and ``consumed_rank_XXXXX.jsonl``
(acknowledged receipts); ``--profile`` records two steps after the warm-up with ``torch.profiler``
and writes the traces after the process group is destroyed. ``--auto-resume`` restores
the newest intact committed checkpoint (model, optimizer shards, EMA, RNG, data cursor).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..config import RunConfig, load_sections
from ..data.device import DeviceLoader
from ..parallel import state as ps
from . import catalog
from . import checkpoint as ckpt
from . import eval_snapshot
from .trainer import Trainer
from ..utils.observe import PhaseTimer, RankLog, StepProfiler, backend_provenance


_LAST_PROFILER = None     # the profiler of the last run(), exported by main() after shutdown


def _all_max(values, device):
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _all_sum(values, device, group=None):
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_initialized():
        dist.all_reduce(t, group=group)
    return t.tolist()


def make_loader(cfg, length, synthetic, seed, dp_rank, dp, prefetch=2, state=None, corpus=None, row_multiple=1):
    from ..data.packing import ConsumedLoader, Packer
    if corpus:
        from ..data.stream import DocumentStream
        documents = DocumentStream(corpus, seed=seed, rank=dp_rank, world=dp)
    else:
        from ..data.synthetic import ListDocuments, joint_pack_documents, tiny_pack_documents, video_pack_documents
        maker = dict(tiny=tiny_pack_documents, joint=joint_pack_documents, video=video_pack_documents)[synthetic]
        docs = []
        for k in range(64):
            docs.extend(maker(cfg, length, seed=seed * 1000 + dp_rank * 100 + k))
        documents = ListDocuments(docs, dict(snapshot="synthetic", seed=seed, epoch=0, rank=dp_rank))
    consumed = (state or {}).get("loader")
    packer = Packer(documents, cfg, length, state=consumed, row_multiple=row_multiple)
    return ConsumedLoader(packer, prefetch=prefetch, state=consumed)


def run(cfg: RunConfig, tp=1, length=8192, steps=10, lr=5e-5, output=Path("runs/default"), training=None,
        synthetic="joint", checkpoint_interval=0, resume=False, global_batch=None, checkpoint_dir=None,
        keep_checkpoints=2, warmup_steps=3, corpus=None, snapshot_interval=0, phase_timing=False, profile=False):
    training = dict(training or {})
    output = Path(output)
    trainer = Trainer(cfg, tp=tp, lr=lr, warmup=int(training.get("lr_warmup_steps", 0)), total_steps=steps,
                      lr_style=training.get("lr_decay_style", "cosine"),
                      ema_decay=float(training.get("renderer_ema_decay", 0.999)),
                      bucket_size=int(training.get("bucket_size", 40_000_000)), seed=int(training.get("seed", 871)))
    st = trainer.state
    rank0 = st.rank == 0
    dp = st.dp
    global_batch = global_batch or int(training.get("global_batch", dp))
    if global_batch % dp:
        raise ValueError(f"global batch {global_batch} must divide DP={dp}")
    grad_accum = global_batch // dp
    ckpt_root = Path(checkpoint_dir) if checkpoint_dir else output / "checkpoints"
    training_state = dict(global_batch=global_batch, seq=length, seed=int(training.get("seed", 871)), synthetic=synthetic,
                          corpus=str(corpus) if corpus else None)
    start_step, data_state = 0, {}
    if resume:
        path = None
        if rank0:
            catalog.remove_incomplete(ckpt_root) if ckpt_root.exists() else None
        if ckpt_root.exists():
            path, _ = catalog.latest(ckpt_root)
        if path:
            start_step = ckpt.load(path, trainer.model, trainer.optimizer, cfg, training_state, data_state, trainer.ema)
            trainer.step_index = start_step
    host_loader = make_loader(cfg, length, synthetic, int(training.get("seed", 871)), st.dp_rank, dp,
                              state=data_state.get("ranks", {}).get(str(st.dp_rank)), corpus=corpus,
                              row_multiple=128 * tp)
    # packs are copied to the GPU on a side stream ahead of their step; the cursor stays acknowledged-only
    loader = DeviceLoader(host_loader, trainer.preparer, prefetch=int(training.get("device_prefetch", 2)))
    if rank0:
        output.mkdir(parents=True, exist_ok=True)
        from ..utils.experiment import source_digest
        params = sum(p.numel() * (tp if getattr(p, "tensor_model_parallel", False) else 1)
                     for p in trainer.model.parameters())
        (output / "run.json").write_text(json.dumps(dict(
            torch=torch.__version__, cuda=torch.version.cuda, world=st.world, tp=tp, dp=dp, global_batch=global_batch,
            grad_accum=grad_accum, sequence_length=length, parameters=params, config=cfg.to_dict(),
            source_digest=source_digest(), start_step=start_step), indent=2))
    rows = []
    step = start_step
    logs = RankLog(output, st.rank)
    profiler = StepProfiler(profile, wait=warmup_steps)
    while step < steps:
        wait0 = time.perf_counter()
        group = [loader.next() for _ in range(grad_accum)]
        data_wait = time.perf_counter() - wait0
        have = [g for g in group if g is not None]
        alive = _all_sum([float(len(have))], trainer.device)[0]
        if alive == 0:
            break
        if not have:
            raise RuntimeError("a DP rank ran out of data before the others; padding graphs are not configured")
        torch.cuda.reset_peak_memory_stats() if trainer.device.type == "cuda" else None
        t0 = time.perf_counter()
        timer = PhaseTimer(trainer.device) if phase_timing else None
        metrics = trainer.train_step([loader.acquire(item) for item in have], prepared=True, phases=timer)
        if trainer.device.type == "cuda":
            torch.cuda.synchronize()
        seconds = time.perf_counter() - t0
        profiler.step()
        for item in have:
            loader.acknowledge(item.receipt)
        logs.acknowledged(step + 1, [item.receipt for item in have])
        phases = metrics.pop("phases", {})
        logs.step(dict(step=step + 1, seconds=seconds, data_wait_seconds=data_wait, phases_ms=phases))
        peak = torch.cuda.max_memory_allocated() / 2 ** 30 if trainer.device.type == "cuda" else 0.0
        names = sorted(phases)
        worst = _all_max([seconds, peak, data_wait] + [phases[k] for k in names], trainer.device)
        seconds, peak, data_wait = worst[:3]
        metrics["data_wait_seconds"] = data_wait
        if names:
            metrics["phases_ms"] = dict(zip(names, worst[3:]))    # max over ranks, like the step time
        step += 1
        tokens = sum(item.receipt["body_tokens"] for item in have)
        total_tokens = _all_sum([float(tokens)], trainer.device, st.dp_group if dp > 1 else None)[0]
        row = dict(step=step, seconds=seconds, tokens_per_second=total_tokens / seconds, peak_gib=peak, **metrics,
                   warmup=step - start_step <= warmup_steps)
        rows.append(row)
        if rank0:
            with (output / "steps.jsonl").open("a") as f:
                f.write(json.dumps(row) + "\n")
            print(json.dumps(row), flush=True)
        if training.get("validation_probes"):
            probes = ckpt.validation_probes(trainer.model, trainer.optimizer)
            (output / "probes").mkdir(parents=True, exist_ok=True)
            torch.save(probes, output / "probes" / f"rank{st.rank}_step_{step:07d}.pt")
        if checkpoint_interval and step % checkpoint_interval == 0:
            states = [None] * st.world if dist.is_initialized() else None
            mine = dict(packer=None, loader=loader.state_dict())
            if dist.is_initialized():
                dist.all_gather_object(states, (st.dp_rank, mine))
                ranks = {str(r): s for r, s in states}
            else:
                ranks = {"0": mine}
            ckpt.save(ckpt_root / f"step_{step:07d}", trainer.model, trainer.optimizer, step, cfg, training_state,
                      dict(ranks=ranks), trainer.ema)
            if rank0:
                catalog.prune(ckpt_root, keep_checkpoints)
        if snapshot_interval and step % snapshot_interval == 0:
            eval_snapshot.save(output / "snapshots" / f"step_{step:07d}", trainer.model, step, cfg, trainer.ema)
    loader.close()
    profiler.stop()
    provenance = backend_provenance()
    provenance.update(rank=st.rank, device_loader=dict(loader.stats) if hasattr(loader, "stats") else None)
    (output / f"backend_rank_{st.rank:05d}.json").write_text(json.dumps(provenance, indent=2))
    global _LAST_PROFILER
    _LAST_PROFILER = profiler
    timed = [r["seconds"] for r in rows if not r["warmup"]] or [r["seconds"] for r in rows]
    if rank0 and rows:
        ordered = sorted(timed)
        summary = dict(steps=len(rows), mean_seconds=statistics.mean(timed), median_seconds=statistics.median(timed),
                       p95_seconds=ordered[min(len(ordered) - 1, int(0.95 * len(ordered)))],
                       content_tokens_per_second=length * global_batch / statistics.median(timed),
                       peak_gib=max(r["peak_gib"] for r in rows), final_loss=rows[-1]["loss"])
        (output / "summary.json").write_text(json.dumps(summary, indent=2))
    return rows


def main(argv=None):
    parser = argparse.ArgumentParser(description="CQ joint pretraining")
    parser.add_argument("--config", required=True)
    parser.add_argument("--output", required=True)
    parser.add_argument("--tp", type=int, default=None)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--sequence-length", type=int, default=None)
    parser.add_argument("--global-batch", type=int, default=None)
    parser.add_argument("--lr", type=float, default=None)
    parser.add_argument("--synthetic", default="joint", choices=("joint", "tiny", "video"))
    parser.add_argument("--corpus", default=None, help="JSONL/Parquet document catalog (instead of synthetic data)")
    parser.add_argument("--checkpoint-interval", type=int, default=0)
    parser.add_argument("--checkpoint-dir", default=None)
    parser.add_argument("--keep-checkpoints", type=int, default=2)
    parser.add_argument("--snapshot-interval", type=int, default=0)
    parser.add_argument("--resume", action="store_true")
    parser.add_argument("--validation-probes", action="store_true",
                        help="write parameter/master/Adam probes after every update (not a speed run)")
    parser.add_argument("--phase-timing", action="store_true",
                        help="CUDA-event forward/backward/optimizer times per step (NVTX ranges for timelines)")
    parser.add_argument("--profile", action="store_true",
                        help="torch.profiler over two steps after the warm-up; traces written after shutdown")
    args = parser.parse_args(argv)
    cfg, training, environment = load_sections(args.config)
    if args.validation_probes:
        training["validation_probes"] = True
    for key, value in environment.items():
        os.environ.setdefault(key, str(value))
    tp = args.tp or int(training.get("tp", 1))
    length = args.sequence_length or int(training.get("sequence_length", 8192))
    lr = args.lr or float(training.get("lr", 5e-5))
    run(cfg, tp=tp, length=length, steps=args.steps, lr=lr, output=Path(args.output), training=training,
        synthetic=args.synthetic, checkpoint_interval=args.checkpoint_interval, resume=args.resume,
        global_batch=args.global_batch, checkpoint_dir=args.checkpoint_dir, keep_checkpoints=args.keep_checkpoints,
        corpus=args.corpus, snapshot_interval=args.snapshot_interval, phase_timing=args.phase_timing,
        profile=args.profile)
    rank = dist.get_rank() if dist.is_initialized() else 0
    if dist.is_initialized():
        dist.barrier()
        ps.destroy()
    profiler = _LAST_PROFILER
    if profiler is not None:     # exported only now: a slow export cannot stall a collective
        profiler.export(Path(args.output) / "profile" / f"rank_{rank:05d}.json")


if __name__ == "__main__":
    main()
