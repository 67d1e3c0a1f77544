"""Run observability: phase timing with NVTX ranges, per-rank logs, backend provenance, profiler.

* ``PhaseTimer``: ``with timer.phase("forward"): ...`` brackets work with CUDA events on the
  current stream and an NVTX range (visible in nsys / ncu timelines); phases may be entered many
  times per step and accumulate. ``collect()`` synchronises once and returns milliseconds per
  phase. The chunked renderer backward enters ``forward`` for each DiT chunk's forward, so that
  time is counted as forward, not backward (reference ``training/train.py:653-698,759-763``).
  A disabled timer (``PhaseTimer(None)``) costs nothing.
* ``RankLog``: per-rank JSON-lines files ``timing_rank_XXXXX.jsonl`` (step seconds, phases, data
  waits) and ``consumed_rank_XXXXX.jsonl`` (the receipts each update acknowledged).
* ``backend_provenance()``: which native libraries this process uses (path and sha256 of the
  kernel library, whether its kernels are enabled, the TP symmetric workspace), device, driver
  and library versions, and the number of native kernel launches so far; the loop writes it to
  ``backend_rank_XXXXX.json`` at exit (reference ``ops/gated_delta_net.py:355-376``).
* ``StepProfiler``: ``torch.profiler`` over steps ``[wait, wait + 1 + active)`` of the loop
  (``--profile``); the trace is only exported by ``export()``, which the loop calls after the
  process group is destroyed, so a slow export can never stall a collective
  (reference ``training/train.py:499-512,866-871``).
"""

from __future__ import annotations

import hashlib
import json
import os
from contextlib import contextmanager, nullcontext
from pathlib import Path

import torch


class PhaseTimer:
    def __init__(self, device, annotate=False):
        self.enabled = device is not None and torch.device(device).type == "cuda"
        self.annotate = annotate   # also open a profiler range per phase (shows on the device timeline)
        self.pairs = []      # (name, start event, end event)

    @contextmanager
    def phase(self, name):
        if not self.enabled:
            yield
            return
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)
        scope = torch.profiler.record_function(name) if self.annotate else nullcontext()
        start.record()
        try:
            with scope:
                yield
        finally:
            end.record()
            torch.cuda.nvtx.range_pop()
            self.pairs.append((name, start, end))

    def collect(self):
        if not self.enabled or not self.pairs:
            return {}
        self.pairs[-1][2].synchronize()
        out = {}
        for name, start, end in self.pairs:
            out[name] = out.get(name, 0.0) + start.elapsed_time(end)
        self.pairs.clear()
        return {k: round(v, 3) for k, v in out.items()}


def phase(timer, name):
    """``timer.phase(name)`` or a no-op context when there is no timer."""
    return timer.phase(name) if timer is not None else nullcontext()


class RankLog:
    def __init__(self, output, rank):
        self.dir = Path(output)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.timing = self.dir / f"timing_rank_{rank:05d}.jsonl"
        self.consumed = self.dir / f"consumed_rank_{rank:05d}.jsonl"

    @staticmethod
    def _append(path, row):
        with path.open("a") as handle:
            handle.write(json.dumps(row) + "\n")

    def step(self, row):
        self._append(self.timing, row)

    def acknowledged(self, step, receipts):
        self._append(self.consumed, dict(step=step, receipts=[{k: v for k, v in r.items() if _plain(v)}
                                                               for r in receipts]))


def _plain(value):
    return isinstance(value, (int, float, str, bool, type(None))) or (
        isinstance(value, (list, tuple)) and all(isinstance(x, (int, float, str, bool)) for x in value))


def _sha256(path):
    digest = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(1 << 20), b""):
            digest.update(block)
    return digest.hexdigest()


def backend_provenance():
    from ..ops import _ext
    info = dict(torch=torch.__version__, cuda_runtime=torch.version.cuda, cuda_available=torch.cuda.is_available())
    lib = _ext.library_path()
    info["kernel_library"] = str(lib) if lib else None
    info["kernel_library_sha256"] = _sha256(lib) if lib and Path(lib).exists() else None
    info["kernels_enabled"] = bool(_ext.cuda_kernels_enabled())
    info["native_launches"] = int(_ext.launches()) if lib else 0
    if torch.cuda.is_available():
        props = torch.cuda.get_device_properties(torch.cuda.current_device())
        info.update(device=props.name, compute_capability=f"{props.major}.{props.minor}",
                    multiprocessors=props.multi_processor_count, memory_gib=round(props.total_memory / 2 ** 30, 1))
        try:
            info["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
        except Exception:  # noqa: BLE001 - NCCL may be absent
            info["nccl"] = None
    from ..parallel import symmetric
    ws = symmetric.workspace()
    info["tp_symmetric_workspace"] = None if ws is None else dict(tp=ws.tp, host_calls=dict(
        all_gather=ws.epoch_ag, reduce_scatter=ws.epoch_rs, statistics=ws.epoch_stat), device_epochs=ws.device_epochs())
    info["deterministic_wgrad"] = os.environ.get("CQB_DETERMINISTIC") == "1"
    return info


class StepProfiler:
    def __init__(self, enabled, wait, active=2):
        self.prof = None
        if enabled:
            from torch.profiler import ProfilerActivity, profile, schedule
            acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
            self.prof = profile(activities=acts, schedule=schedule(wait=wait, warmup=1, active=active, repeat=1),
                                record_shapes=True, profile_memory=True)
            self.prof.__enter__()

    def step(self):
        if self.prof is not None:
            self.prof.step()

    def stop(self):
        if self.prof is not None:
            self.prof.__exit__(None, None, None)

    def export(self, path):
        """Write the chrome trace and a per-kernel table (after the process group is gone)."""
        if self.prof is None:
            return None
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        self.prof.export_chrome_trace(str(path))
        table = self.prof.key_averages().table(sort_by="self_cuda_time_total" if torch.cuda.is_available()
                                               else "self_cpu_time_total", row_limit=60)
        path.with_suffix(".txt").write_text(table)
        return path
