"""Training runtime: the public ``Trainer`` API and the ``python -m cq_pretrain_b200.train.trainer`` CLI.

One update (reference ``training/train.py:587-780``): zero gradients; for each accumulation
micro-batch copy the pinned host batch to the device, run ``JointModel.forward``, compose the
weighted losses with DP scales and backpropagate (through the chunked renderer schedule when
the batch plans DiT micro-batches); reduce gradients (TP-sum replicated, DP reduce-scatter),
clip, AdamW-update the owned shards, all-gather parameters, update the renderer EMA; read the
loss back to the host. A non-finite loss or skipped update raises ``FloatingPointError``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import time
from contextlib import nullcontext
from pathlib import Path

import torch
import torch.distributed as dist

from ..config import RunConfig, load_sections
from ..data.preparer import DevicePreparer
from ..models.joint import JointModel
from ..models.qwen35 import cast_for_training
from ..parallel import state as ps
from ..parallel.ddp import DistributedOptimizer
from .ema import RendererEMA
from .graphed import RendererGraphs, graphs_enabled
from .loss import compose_losses, scales_from_counts
from .renderer_schedule import backward_deferred_renderer
from .schedule import learning_rate
from ..utils.observe import phase


def build_model(cfg, device, seed=871, dtype=torch.bfloat16):
    torch.manual_seed(seed)
    if device.type == "cuda":
        torch.cuda.manual_seed_all(seed)
    with torch.device(device):
        model = JointModel(cfg)
    if dtype != torch.float32:
        cast_for_training(model, dtype)
    model.train()
    return model


class Trainer:
    """Owns model, optimizer, EMA and preparer for one rank; ``train_step`` runs one update."""

    def __init__(self, cfg: RunConfig, tp=1, lr=5e-5, warmup=0, total_steps=0, lr_style="cosine",
                 ema_decay=0.999, bucket_size=40_000_000, overlap=None, seed=871, device=None,
                 dtype=torch.bfloat16, fused_tp=True):
        self.state = ps.initialize(tp) if ps.state().tp != tp or not dist.is_initialized() else ps.state()
        self.device = torch.device(device) if device is not None else self.state.device
        cfg.validate(tp)
        self.cfg = cfg
        self.lr, self.warmup, self.total_steps, self.lr_style = lr, warmup, total_steps, lr_style
        self.model = build_model(cfg, self.device, seed, dtype)
        if overlap is None:   # launch each DP bucket's reduce-scatter during backward once it is complete
            overlap = self.state.dp > 1
        self.optimizer = DistributedOptimizer(self.model, lr, bucket_size=bucket_size, overlap=overlap)
        self.ema = RendererEMA(self.model, self.optimizer, ema_decay) if ema_decay else None
        self.preparer = DevicePreparer(cfg, self.device, dtype)
        self.step_index = 0
        # the DiT chunk (forward + backward) replays as a CUDA graph once its geometry repeats
        # (at TP > 1 only with the fused TP kernels: captured NCCL collectives measured slower than eager)
        use_graphs = graphs_enabled(cfg, self.device, tp) and (tp == 1 or fused_tp)
        self.renderer_graphs = RendererGraphs(self.optimizer) if use_graphs else None
        if tp > 1 and fused_tp and self.device.type == "cuda":
            from ..parallel import symmetric
            symmetric.enable()

    def close(self):
        """Release the captured renderer graphs (call before ``parallel.state.destroy``)."""
        if self.renderer_graphs is not None:
            self.renderer_graphs.release()

    def _micro(self, batch, scales, backward_scale, timer=None):
        deferred = batch.generation is not None and (bool(batch.generation.microbatches)
                                                     or self.renderer_graphs is not None)
        with phase(timer, "forward"):
            out = self.model(batch, compute_image_loss=not deferred)
            losses = compose_losses(out, self.cfg, scales)
        if deferred:
            image_factor = self.cfg.image_weight * scales[1]
            losses = backward_deferred_renderer(self.model, batch, losses, backward_scale, self.optimizer,
                                                image_factor=image_factor, timer=timer, graphs=self.renderer_graphs)
        else:
            with phase(timer, "backward"):
                (losses["loss"] * backward_scale).backward()
        return losses

    def train_step(self, micro_batches, timing=False, prepared=False, phases=None):
        """``micro_batches``: list of (pinned host batch, receipt). Returns host-side metrics of the update.

        The step copies every micro-batch to the device, runs the update, and reads the loss back.
        With ``prepared=True`` the batches are already on the device (``data.device.DeviceLoader``
        copied them on its side stream). With ``timing`` it also reports ``compute_ms``: CUDA-event
        time from after the copies were issued to the end of the optimizer/EMA work (excludes the
        host->device and device->host I/O). With a ``phases`` timer (``utils.observe.PhaseTimer``)
        it also reports ``phases``: forward / backward / optimizer milliseconds (NVTX-ranged).
        """
        if prepared:
            device_batches = [batch for batch, _ in micro_batches]
        else:
            device_batches = [self.preparer(host, receipt, non_blocking=True) for host, receipt in micro_batches]
        events = None
        if timing and self.device.type == "cuda":
            events = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            events[0].record()
        n_text = sum(int(b.text_indices.numel()) for b, _ in micro_batches)
        n_img = sum(b.generation_image_count for b, _ in micro_batches)
        if self.state.dp > 1:
            # before the gradient zeroing: the host waits for this small collective only
            counts = torch.tensor([float(n_text), float(n_img)], dtype=torch.float64, device=self.device)
            dist.all_reduce(counts, group=self.state.dp_group)
            total_text, total_img = counts.tolist()
        else:   # nothing to combine: no device round trip (it would wait for the queued work)
            total_text, total_img = float(n_text), float(n_img)
        self.optimizer.zero_grad()
        dp = self.state.dp
        accumulated = torch.zeros(3, dtype=torch.float32, device=self.device)
        ga = len(micro_batches)
        for i, host in enumerate(device_batches):
            # Global-average weights: each micro-batch's mean losses count by its share of all
            # text targets / generation images across DP ranks and accumulation steps.
            scales = scales_from_counts(int(host.text_indices.numel()), host.generation_image_count, total_text,
                                        total_img, dp)
            ctx = self.optimizer.no_sync() if i + 1 < ga else nullcontext()
            with ctx:
                losses = self._micro(host, scales, 1.0, phases)
            accumulated += torch.stack((losses["loss"].detach().float(),
                                        losses["text_loss"].detach().float() * scales[0],
                                        losses["image_loss"].detach().float() * scales[1]))
        with phase(phases, "optimizer"):
            self.optimizer.finish_grad_sync()
            lr = learning_rate(self.step_index, self.lr, self.warmup, self.total_steps, self.lr_style)
            updated, norm = self.optimizer.step(lr)
            if self.ema is not None:
                self.ema.update()
        self.step_index += 1
        if events is not None:
            events[1].record()
        values = torch.cat((accumulated, norm.reshape(1).float(), updated.reshape(1).float())).cpu()
        loss, text, image, gnorm, updated = values.tolist()
        if not updated or not math.isfinite(loss):
            raise FloatingPointError(f"non-finite loss or skipped update at step {self.step_index}")
        out = dict(loss=loss, text_loss=text, image_loss=image, grad_norm=gnorm, lr=lr)
        if events is not None:
            out["compute_ms"] = events[0].elapsed_time(events[1])
        if phases is not None:
            out["phases"] = phases.collect()
        return out


def main(argv=None):
    parser = argparse.ArgumentParser(description="CQ joint pretraining on synthetic or corpus data")
    parser.add_argument("--config", required=True)
    parser.add_argument("--output", required=True)
    parser.add_argument("--tp", type=int, default=None)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--sequence-length", type=int, default=None)
    parser.add_argument("--global-batch", type=int, default=None)
    parser.add_argument("--lr", type=float, default=None)
    parser.add_argument("--synthetic", default="joint", choices=("joint", "tiny", "video"))
    parser.add_argument("--checkpoint-interval", type=int, default=0)
    parser.add_argument("--resume", action="store_true")
    args = parser.parse_args(argv)
    cfg, training, environment = load_sections(args.config)
    for key, value in environment.items():
        os.environ.setdefault(key, str(value))
    tp = args.tp or int(training.get("tp", 1))
    length = args.sequence_length or int(training.get("sequence_length", 8192))
    lr = args.lr or float(training.get("lr", 5e-5))
    from .loop import run
    run(cfg, tp=tp, length=length, steps=args.steps, lr=lr, output=Path(args.output), training=training,
        synthetic=args.synthetic, checkpoint_interval=args.checkpoint_interval, resume=args.resume,
        global_batch=args.global_batch)


if __name__ == "__main__":
    main()
