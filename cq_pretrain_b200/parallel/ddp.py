"""Data parallelism with a ZeRO-1 distributed AdamW optimizer.

Layout (reference ``distributed/megatron.py:210-240`` used Megatron DDP + distributed optimizer):

* parameters of one dtype live as views of one flat buffer; gradients accumulate in a flat
  FP32 ``main_grad`` buffer with the same layout (``gradient_accumulation_fusion``);
* the buffers are cut into buckets (about ``bucket_size`` elements, reverse registration
  order = backward order), each padded to a multiple of the DP size;
* each bucket is reduce-scattered over DP in FP32 (averaged), so rank ``r`` owns shard ``r``
  of every bucket; AdamW updates the FP32 master copy of the owned shard; the updated shard
  is cast and all-gathered back into the parameter buffer;
* under sequence-parallel TP, parameters replicated across the TP group (norms, biases of
  row-parallel linears, DiT modulation/time layers) receive partial gradients on each TP
  rank; their gradients are summed over TP (one coalesced all-reduce) before DP reduction
  (reference ``distributed/megatron.py:243-266`` did this for the Q/K norms); parameters marked
  ``tp_duplicate`` (the vision tower's norms and biases under vision TP, which runs on replicated
  activations) already hold the full gradient on every TP rank and skip that sum;
* bucket reduce-scatters are dispatched in one fixed index order on every rank, so ranks
  whose batches skip a branch (no images, no text) still issue identical collective
  sequences (reference ``distributed/communication.py:12-116``). With ``overlap=True`` a
  bucket launches during backward once every parameter reported its gradient (counts learned
  on the first step; ``suspend_readiness`` keeps non-final DiT chunks from triggering it).
* with ``overlap_param_gather`` (default under NCCL with DP > 1; the reference's
  ``overlap_param_gather=True``) the bf16 parameter all-gather after the update is left running:
  buckets are issued in forward order and forward pre-hooks make the compute stream wait for a
  bucket only when the first module reading it is about to run.

The grad-norm clip (1.0), betas (0.9, 0.95), eps 1e-8, decoupled weight decay (not on
biases / 1-D parameters) and ``min_lr = 0.1 lr`` follow the reference optimizer config. On
CUDA the update of all owned shards is one multi-tensor kernel (``csrc/optim.cu``) that also
writes the updated parameters in their training dtype, and the global gradient norm is one
multi-tensor reduction.
"""

from __future__ import annotations

import math
from contextlib import contextmanager

import torch
import torch.distributed as dist

from ..ops import _ext
from . import state as ps


class Bucket:
    def __init__(self, index, group, start, end, params):
        self.index, self.group, self.start, self.end = index, group, start, end
        self.params = params
        self.handle = None
        self.launched = False
        self.counts = {}
        self.gather = None        # pending parameter all-gather (work handle, source shard)


class ParamGroup:
    """One dtype (and replication class): flat param + fp32 grad buffers."""

    def __init__(self, name, dtype, params, device, dp, bucket_size, align=128):
        self.name, self.dtype, self.params = name, dtype, params
        offsets, cursor = {}, 0
        bucket_bounds, bucket_start, bucket_params, current = [], 0, [], []
        unit = dp * align
        for p in params:
            cursor = -(-cursor // 64) * 64  # 128-byte aligned parameter views (TMA / vector loads)
            offsets[p] = cursor
            cursor += p.numel()
            current.append(p)
            if cursor - bucket_start >= bucket_size:
                end = -(-cursor // unit) * unit
                bucket_bounds.append((bucket_start, end, current))
                cursor = bucket_start = end
                current = []
        if current:
            end = -(-cursor // unit) * unit
            bucket_bounds.append((bucket_start, end, current))
            cursor = end
        self.numel = cursor
        self.param_buffer = torch.zeros(cursor, dtype=dtype, device=device)
        self.grad_buffer = torch.zeros(cursor, dtype=torch.float32, device=device)
        self.offsets = offsets
        self.bucket_bounds = bucket_bounds
        for p in params:
            o = offsets[p]
            view = self.param_buffer[o:o + p.numel()].view_as(p)
            view.copy_(p.data)
            p.data = view
            p.main_grad = self.grad_buffer[o:o + p.numel()].view_as(p)


class DistributedOptimizer:
    def __init__(self, model, lr, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8, clip_grad=1.0,
                 bucket_size=40_000_000, overlap=False, ema_prefix=None, ema_decay=None, overlap_param_gather=None):
        st = ps.state()
        self.model = model
        self.lr, self.weight_decay, self.betas, self.eps, self.clip_grad = lr, weight_decay, betas, eps, clip_grad
        self.dp, self.dp_rank, self.dp_group = st.dp, st.dp_rank, st.dp_group
        self.tp, self.tp_group, self.tp_rank = st.tp, st.tp_group, st.tp_rank
        self.overlap = overlap
        self.ema, self.ema_fused = None, False
        named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
        self.names = {p: n for n, p in named}
        device = named[0][1].device
        groups: dict = {}
        for n, p in reversed(named):
            plain = self.tp > 1 and not getattr(p, "tensor_model_parallel", False)
            duplicate = plain and getattr(p, "tp_duplicate", False)
            key = (p.dtype, plain and not duplicate, duplicate)
            groups.setdefault(key, []).append(p)
        self.groups = []
        for (dtype, replicated, duplicate), params in sorted(groups.items(),
                                                             key=lambda kv: (kv[0][1], kv[0][2], str(kv[0][0]))):
            suffix = "-replicated" if replicated else "-duplicate" if duplicate else ""
            g = ParamGroup(f"{str(dtype).split('.')[-1]}{suffix}", dtype, params, device, self.dp, bucket_size)
            g.replicated, g.duplicate = replicated, duplicate
            self.groups.append(g)
        self.buckets = []
        for g in self.groups:
            for start, end, params in g.bucket_bounds:
                self.buckets.append(Bucket(len(self.buckets), g, start, end, params))
        self.param_bucket = {p: b for b in self.buckets for p in b.params}
        # Owned shard state (fp32 master, exp_avg, exp_avg_sq, decay mask, ema shadow).
        self.shards = []
        for b in self.buckets:
            n = (b.end - b.start) // self.dp
            lo = b.start + self.dp_rank * n
            master = b.group.param_buffer[lo:lo + n].float().clone()
            decay = torch.zeros(n, dtype=torch.uint8, device=device)
            ema_mask = torch.zeros(n, dtype=torch.bool, device=device)
            for p in b.params:
                o = b.group.offsets[p]
                a, e = max(o, lo), min(o + p.numel(), lo + n)
                if a < e:
                    name = self.names[p]
                    if p.dim() > 1 and not name.endswith(".bias"):
                        decay[a - lo:e - lo] = 1
                    if ema_prefix and name.startswith(ema_prefix):
                        ema_mask[a - lo:e - lo] = True
            self.shards.append(dict(bucket=b, lo=lo, n=n, master=master, exp_avg=torch.zeros_like(master),
                                    exp_avg_sq=torch.zeros_like(master), decay=decay, ema_mask=ema_mask))
        self.step_count = 0
        self.learned = False
        self.suspended = 0
        self.next_bucket = 0
        if overlap_param_gather is None:
            overlap_param_gather = self.dp > 1 and dist.get_backend(self.dp_group) == "nccl"
        self.overlap_param_gather = bool(overlap_param_gather)
        self._gather_hooks = self._install_gather_hooks(model) if self.overlap_param_gather else []
        for p in self.names:
            p._grad_ready = self._mark
            if not getattr(p, "_direct_main_grad", False):
                p.register_post_accumulate_grad_hook(self._accumulate_hook)

    # ---- gradient flow ---------------------------------------------------------------------------
    def _accumulate_hook(self, p):
        if p.grad is not None:
            p.main_grad.add_(p.grad.view_as(p.main_grad))
            p.grad = None
        self._mark(p)

    def _mark(self, p):
        b = self.param_bucket.get(p)
        if b is None:
            return
        if b.launched:
            raise RuntimeError(f"gradient of {self.names[p]} arrived after its bucket reduce-scatter started")
        if getattr(self, "_recorded", None) is not None:
            self._recorded.append(p)
            return
        if self.suspended:
            return
        b.counts[p] = b.counts.get(p, 0) + 1
        if self.overlap and self.learned and not b.group.replicated:
            self._dispatch_ready()

    def _bucket_ready(self, b):
        return all(b.counts.get(p, 0) >= self.expected.get(p, 1) for p in b.params)

    def _dispatch_ready(self):
        while self.next_bucket < len(self.buckets):
            b = self.buckets[self.next_bucket]
            if b.group.replicated or not self._bucket_ready(b):
                return
            self._launch(b)

    def _launch(self, b):
        n = (b.end - b.start) // self.dp
        full = b.group.grad_buffer[b.start:b.end]
        if self.dp > 1:
            if dist.get_backend(self.dp_group) == "gloo":   # CPU tests: gloo has no reduce-scatter
                b.handle = dist.all_reduce(full, group=self.dp_group, async_op=True)
            else:
                out = full[self.dp_rank * n:(self.dp_rank + 1) * n]
                b.handle = dist.reduce_scatter_tensor(out, full, op=dist.ReduceOp.SUM, group=self.dp_group,
                                                      async_op=True)
        b.launched = True
        self.next_bucket = max(self.next_bucket, b.index + 1)

    def start_recording(self):
        """Readiness marks from now on are recorded instead of counted (a CUDA-graph capture,
        whose backward runs again on every replay); ``stop_recording`` returns them in order."""
        self._recorded = []

    def stop_recording(self):
        marks, self._recorded = self._recorded, None
        return marks or []

    @contextmanager
    def suspend_readiness(self):
        """Gradients accumulate but do not count toward bucket readiness (non-final DiT chunks)."""
        self.suspended += 1
        try:
            yield
        finally:
            self.suspended -= 1

    @contextmanager
    def no_sync(self):
        """Gradient accumulation micro-batch: accumulate only; nothing is reduced."""
        previous = self.overlap
        self.overlap = False
        self.suspended += 1
        try:
            yield
        finally:
            self.suspended -= 1
            self.overlap = previous

    def zero_grad(self):
        for g in self.groups:
            g.grad_buffer.zero_()
        for b in self.buckets:
            b.launched, b.handle, b.counts = False, None, {}
        self.next_bucket = 0

    def finish_grad_sync(self):
        """TP-sum replicated grads, then reduce-scatter every bucket over DP in fixed order."""
        if not self.learned:
            self.expected = {p: max(1, b.counts.get(p, 1)) for b in self.buckets for p in b.params}
            self.learned = True
        if self.tp > 1:
            for g in self.groups:
                if g.replicated:
                    dist.all_reduce(g.grad_buffer, group=self.tp_group)
        for b in self.buckets:
            if not b.launched:
                self._launch(b)
        for b in self.buckets:
            if b.handle is not None:
                b.handle.wait()
                b.handle = None

    # ---- optimizer -----------------------------------------------------------------------------
    def _grad_shard(self, s):
        b = s["bucket"]
        return b.group.grad_buffer[s["lo"]:s["lo"] + s["n"]]

    def _use_kernels(self):
        return self.shards[0]["master"].is_cuda and _ext.cuda_kernels_enabled() and _ext.has("adamw_step")

    def grad_norm(self):
        counted = [self._grad_shard(s) for s in self.shards
                   if not ((s["bucket"].group.replicated or s["bucket"].group.duplicate) and self.tp_rank != 0)
                   and s["n"]]
        if counted and self._use_kernels():
            total = _ext.ops().sum_squares(counted)   # one multi-tensor pass, fixed reduction order
        else:
            total = torch.zeros((), dtype=torch.float32, device=self.shards[0]["master"].device)
            for g in counted:
                total += g.float().square().sum()
        if self.dp > 1:
            dist.all_reduce(total, group=self.dp_group)
        if self.tp > 1:
            dist.all_reduce(total, group=self.tp_group)
        return total.sqrt()

    @torch.no_grad()
    def step(self, lr=None, ema_decay=None):
        """Average, clip, AdamW-update owned shards, optional EMA, then all-gather parameters
        (asynchronously when ``overlap_param_gather``: the next forward waits per bucket)."""
        self.wait_params()      # the update writes into buffers a pending gather may still fill
        lr = self.lr if lr is None else lr
        self.step_count += 1
        scale = 1.0 / self.dp
        norm = self.grad_norm() * scale
        coef = torch.clamp(self.clip_grad / (norm + 1e-6), max=1.0) if self.clip_grad else torch.ones_like(norm)
        finite = torch.isfinite(norm)
        b1, b2 = self.betas
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        gscale = (coef * scale).float().reshape(())
        if self._use_kernels():
            # one launch: scale, moments, decoupled decay, update, the parameter write-back and (when
            # a renderer EMA is attached) the shadow lerp toward the updated masters
            lists = self._kernel_lists()
            _ext.ops().adamw_step(*lists[:6], gscale, lr, b1, b2, self.eps, self.weight_decay, bc1, bc2,
                                  lists[6], 1.0 - self.ema.decay if self.ema is not None else 0.0)
            self.ema_fused = self.ema is not None
        else:
            grads = [self._grad_shard(s) for s in self.shards]
            published = [s["bucket"].group.param_buffer[s["lo"]:s["lo"] + s["n"]] for s in self.shards]
            for s, g, out in zip(self.shards, grads, published):
                g = g * gscale
                m, v, p = s["exp_avg"], s["exp_avg_sq"], s["master"]
                m.mul_(b1).add_(g, alpha=1 - b1)
                v.mul_(b2).addcmul_(g, g, value=1 - b2)
                update = (m / bc1) / ((v / bc2).sqrt() + self.eps)
                p.mul_(1 - lr * self.weight_decay * s["decay"].float())
                p.add_(update, alpha=-lr)
                out.copy_(p)
        self.all_gather_params(blocking=not self.overlap_param_gather)
        return finite, norm

    def attach_ema(self, ema):
        """Let the AdamW kernel update ``ema``'s shadows (``shadow += (1 - decay)(master - shadow)``)."""
        self.ema, self.ema_fused = ema, False

    def _kernel_lists(self):
        """Per-shard tensors for the AdamW kernel, split at the EMA slices so that each renderer
        slice carries its shadow (an empty tensor marks slices without one). Every entry is a view
        of a persistent buffer, so the lists are built once (thousands of slices: tens of ms of
        host time per step otherwise) and rebuilt only when another EMA or shadow set is attached."""
        ema = getattr(self, "ema", None)
        key = (id(ema), tuple(map(id, ema.shadows)) if ema is not None else ())
        cached = getattr(self, "_lists_cache", None)
        if cached is not None and cached[0] == key:
            return cached[1]
        grads = [self._grad_shard(s) for s in self.shards]
        published = [s["bucket"].group.param_buffer[s["lo"]:s["lo"] + s["n"]] for s in self.shards]
        ranges = {}
        if ema is not None:
            for (si, a, b), shadow in zip(ema.index, ema.shadows):
                ranges.setdefault(si, []).append((a, b, shadow))
        out = [[] for _ in range(7)]
        none = self.shards[0]["master"].new_empty(0)
        for si, (s, g, pub) in enumerate(zip(self.shards, grads, published)):
            tensors = (s["master"], g, s["exp_avg"], s["exp_avg_sq"], s["decay"], pub)
            cuts, cursor = [], 0
            for a, b, shadow in sorted(ranges.get(si, []), key=lambda r: r[0]):
                if a > cursor:
                    cuts.append((cursor, a, none))
                cuts.append((a, b, shadow))
                cursor = b
            if cursor < s["n"]:
                cuts.append((cursor, s["n"], none))
            for a, b, shadow in cuts:
                for lst, t in zip(out, tensors):
                    lst.append(t[a:b])
                out[6].append(shadow)
        self._lists_cache = (key, out)
        return out

    def all_gather_params(self, blocking=True):
        """Publish every rank's updated shards to all DP ranks.

        Buckets are issued in forward order (the reverse of the bucket order, which follows the
        backward), so the first layers' parameters arrive first. With ``blocking=False`` the
        gathers stay pending: the forward pre-hooks make the compute stream wait for a bucket
        right before the first module that reads it, and ``wait_params`` waits for the rest."""
        if self.dp == 1:
            return
        self.wait_params()
        for b in reversed(self.buckets):
            n = (b.end - b.start) // self.dp
            full = b.group.param_buffer[b.start:b.end]
            mine = full[self.dp_rank * n:(self.dp_rank + 1) * n].clone()
            if dist.get_backend(self.dp_group) == "gloo":
                dist.all_gather(list(full.split(n)), mine, group=self.dp_group)
                continue
            b.gather = (dist.all_gather_into_tensor(full, mine, group=self.dp_group, async_op=True), mine)
        if blocking:
            self.wait_params()

    def _await(self, buckets):
        for b in buckets:
            if b.gather is not None:
                b.gather[0].wait()      # stream-side wait: the host does not block
                b.gather = None

    def wait_params(self):
        """Make the current stream wait for every pending parameter all-gather."""
        self._await(self.buckets)

    def _install_gather_hooks(self, model):
        """Forward pre-hooks on the outermost modules whose parameters span at most two buckets
        (and on every leaf module): each waits for its parameters' buckets. Parameters no hooked
        module covers are waited for when the model itself is called."""
        covered, hooks = set(), []

        def add(module, buckets):
            hooks.append(module.register_forward_pre_hook(lambda m, args, bs=tuple(buckets): self._await(bs)))

        def visit(module):
            params = [p for p in module.parameters() if p in self.param_bucket]
            buckets = sorted({self.param_bucket[p].index for p in params})
            children = list(module.children())
            if buckets and module is not model and (not children or len(buckets) <= 2):
                add(module, [self.buckets[i] for i in buckets])
                covered.update(params)
                return
            for child in children:
                visit(child)
            direct = [p for p in module.parameters(recurse=False) if p in self.param_bucket]
            if direct and module is not model:
                add(module, sorted({self.param_bucket[p] for p in direct}, key=lambda b: b.index))
                covered.update(direct)

        visit(model)
        rest = sorted({self.param_bucket[p] for p in self.param_bucket if p not in covered}, key=lambda b: b.index)
        if rest:
            add(model, rest)
        return hooks

    # ---- checkpoint -------------------------------------------------------------------------
    def state_dict(self):
        return dict(step=self.step_count,
                    shards=[dict(master=s["master"], exp_avg=s["exp_avg"], exp_avg_sq=s["exp_avg_sq"]) for s in self.shards],
                    layout=[(s["bucket"].group.name, s["lo"], s["n"]) for s in self.shards])

    @torch.no_grad()
    def load_state_dict(self, state):
        layout = [(s["bucket"].group.name, s["lo"], s["n"]) for s in self.shards]
        if [tuple(x) for x in state["layout"]] != layout:
            raise ValueError("optimizer shard layout differs from the checkpoint")
        for s, saved in zip(self.shards, state["shards"]):
            for key in ("master", "exp_avg", "exp_avg_sq"):
                s[key].copy_(saved[key])
            b = s["bucket"]
            b.group.param_buffer[s["lo"]:s["lo"] + s["n"]].copy_(s["master"])
        self.step_count = state["step"]
        self.all_gather_params(blocking=True)
