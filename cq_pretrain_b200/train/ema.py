"""Renderer-only FP32 EMA kept on the distributed optimizer's master shards.

``shadow += (1 - decay) (master - shadow)`` on the slice of every owned shard that belongs
to ``renderer.*`` parameters: no collectives, and no rank holds a full DiT copy (reference
``training/ema.py:17-119``). On CUDA the lerp runs inside the optimizer's AdamW kernel (the
updated master is still in registers); ``update`` then only counts the step. ``average_parameters`` temporarily installs the shadows into the
masters and republishes the parameters (all-gather), restoring the online weights after.
"""

from __future__ import annotations

import math
from contextlib import contextmanager

import torch
import torch.distributed as dist


class RendererEMA:
    schema = "fp32_optimizer_shards_v1"

    @torch.no_grad()
    def __init__(self, model, optimizer, decay=0.9999, prefix="renderer."):
        if not math.isfinite(decay) or not 0 <= decay < 1:
            raise ValueError("EMA decay must be finite and in [0, 1)")
        self.decay, self.num_updates, self.active = float(decay), 0, False
        self.optimizer, self.prefix = optimizer, prefix
        names = {p: n for n, p in model.named_parameters() if n.startswith(prefix) and p.requires_grad}
        if not names:
            raise ValueError("renderer EMA requires trainable renderer parameters")
        self.layout, self.index, self.shadows = [], [], []
        for si, shard in enumerate(optimizer.shards):
            b = shard["bucket"]
            for p in b.params:
                if p not in names:
                    continue
                o = b.group.offsets[p]
                a, e = max(o, shard["lo"]), min(o + p.numel(), shard["lo"] + shard["n"])
                if a < e:
                    self.layout.append(dict(name=names[p], start=a - o, end=e - o))
                    self.index.append((si, a - shard["lo"], e - shard["lo"]))
                    self.shadows.append(shard["master"][a - shard["lo"]:e - shard["lo"]].clone())
        covered = torch.tensor(sum(s.numel() for s in self.shadows), dtype=torch.int64,
                               device=optimizer.shards[0]["master"].device)
        if optimizer.dp > 1:
            dist.all_reduce(covered, group=optimizer.dp_group)
        if int(covered) != sum(p.numel() for p in names):
            raise ValueError("EMA shards do not cover the renderer exactly once")
        if hasattr(optimizer, "attach_ema"):
            optimizer.attach_ema(self)    # the AdamW kernel lerps the shadows in its own pass

    def masters(self):
        return [self.optimizer.shards[si]["master"][a:b] for si, a, b in self.index]

    @torch.no_grad()
    def update(self):
        if self.active:
            raise RuntimeError("cannot update EMA while EMA weights are installed")
        if getattr(self.optimizer, "ema_fused", False):
            self.optimizer.ema_fused = False      # the optimizer step already lerped the shadows
        elif self.shadows:
            torch._foreach_lerp_(self.shadows, self.masters(), 1.0 - self.decay)
        self.num_updates += 1

    def metadata(self):
        return dict(schema=self.schema, module="renderer", decay=self.decay, num_updates=self.num_updates,
                    dtype="float32")

    def state_dict(self):
        if self.active:
            raise RuntimeError("checkpointing during an EMA swap is forbidden")
        return dict(**self.metadata(), layout=self.layout, shadows=self.shadows)

    @torch.no_grad()
    def load_state_dict(self, state):
        expected = self.metadata()
        expected.pop("num_updates")
        if any(state.get(k) != v for k, v in expected.items()) or state.get("layout") != self.layout:
            raise ValueError("EMA decay, module, dtype or shard layout differs")
        if len(state["shadows"]) != len(self.shadows):
            raise ValueError("EMA shard count differs")
        for value, target in zip(state["shadows"], self.shadows):
            if value.dtype != torch.float32 or value.shape != target.shape:
                raise ValueError("EMA tensor dtype/shape differs")
            target.copy_(value)
        self.num_updates = int(state["num_updates"])

    @torch.no_grad()
    def _publish(self):
        self.optimizer.wait_params()
        for s in self.optimizer.shards:
            b = s["bucket"]
            b.group.param_buffer[s["lo"]:s["lo"] + s["n"]].copy_(s["master"])
        self.optimizer.all_gather_params()

    @contextmanager
    def average_parameters(self):
        if self.active:
            raise RuntimeError("nested EMA swaps are forbidden")
        masters = self.masters()
        online = [m.clone() for m in masters]
        self.active = True
        try:
            with torch.no_grad():
                for m, s in zip(masters, self.shadows):
                    m.copy_(s)
                self._publish()
            yield self
        finally:
            with torch.no_grad():
                for m, v in zip(masters, online):
                    m.copy_(v)
                self._publish()
            self.active = False
