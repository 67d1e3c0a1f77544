"""Staged, bounded tuning matrix on one node (reference ``tune64.py:16-118``).

``python -m cq_pretrain_b200.launch.tune --plan plan.json`` runs each stage of the plan as its own
training job (``torch.distributed.run`` over the node's GPUs, own process group) and records the
outcome in ``<output>/progress.json``. A plan::

    {"output": "runs/tune", "nproc": 8, "memory_guard_gib": 150,
     "common_args": ["--config", "cq_pretrain_b200/configs/qwen35_2b_wan.yaml", "--steps", "20"],
     "defaults": {"tp": 2},
     "stages": [
        {"name": "base"},
        {"name": "gb64", "knobs": {"global_batch": 64}},
        {"name": "best-tp4", "select_from": ["base", "gb64"], "knobs": {"tp": 4},
         "requires_success": ["base"], "optional": true, "timeout_seconds": 1800}]}

Knobs become ``--name value`` flags (``True`` -> bare flag). ``select_from`` starts from the knobs
of the fastest successful listed stage (median tokens/s of ``summary.json``) whose peak memory
stayed under the guard. A stage is stopped (SIGTERM to its process group, SIGKILL after 15 s)
when a step reports peak memory above the guard or its deadline passes; a required stage that
fails stops the matrix, and an unexplained failure (not memory) stops it too instead of being
retried. ``<output>/stop_after_current_stage`` ends the matrix at the next stage boundary.
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys
import time
from pathlib import Path

from ..utils.files import atomic_json


def _score(folder):
    path = folder / "summary.json"
    if not path.exists():
        return None
    summary = json.loads(path.read_text())
    return summary.get("content_tokens_per_second"), summary.get("peak_gib", 0.0)


def best(root, names, guard):
    candidates = []
    for name in names:
        folder = root / name
        exit_file = folder / "exit.json"
        if not exit_file.exists() or json.loads(exit_file.read_text())["returncode"] != 0:
            continue
        score = _score(folder)
        if score is None or score[0] is None or score[1] > guard:
            continue
        candidates.append((score[0], name))
    if not candidates:
        raise RuntimeError(f"no successful candidate under the {guard} GiB memory guard among {names}")
    return max(candidates)[1]


def argv_for(knobs, common):
    argv = list(common)
    for name, value in knobs.items():
        option = "--" + name.replace("_", "-")
        if value is True:
            argv.append(option)
        elif value is not False and value is not None:
            argv.append(option)
            argv.extend(str(v) for v in (value if isinstance(value, list) else [value]))
    return argv


def _memory_breach(folder, guard):
    steps = folder / "steps.jsonl"
    if not steps.exists():
        return None
    lines = [line for line in steps.read_text().splitlines(keepends=True) if line.endswith("\n")]
    for line in lines:
        row = json.loads(line)
        if row.get("peak_gib", 0.0) > guard:
            return dict(memory=dict(step=row.get("step"), peak_gib=row["peak_gib"], limit_gib=guard))
    return None


def _watch(process, folder, guard, deadline, poll):
    """Wait for the job; stop it on memory-guard breach or deadline. Returns the rejection reason."""
    reason = None
    while process.poll() is None:
        reason = _memory_breach(folder, guard)
        if reason is None and time.monotonic() > deadline:
            reason = dict(deadline=True)
        if reason is not None:
            try:
                os.killpg(process.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
            try:
                process.wait(timeout=15)
            except subprocess.TimeoutExpired:
                os.killpg(process.pid, signal.SIGKILL)
                process.wait()
            break
        time.sleep(poll)
    return reason or _memory_breach(folder, guard)   # a job that ended over the guard is rejected too


def run(plan, poll=2.0):
    root = Path(plan["output"])
    root.mkdir(parents=True, exist_ok=True)
    guard = float(plan.get("memory_guard_gib", 150.0))
    outcomes = []
    for stage in plan["stages"]:
        if (root / "stop_after_current_stage").exists():
            break
        missing = [n for n in stage.get("requires_success", [])
                   if not any(o["name"] == n and o.get("passed") for o in outcomes)]
        if missing:
            outcomes.append(dict(name=stage["name"], passed=False, skipped=True, requires=missing))
            atomic_json(root / "progress.json", dict(completed=outcomes))
            continue
        folder = root / stage["name"]
        folder.mkdir(parents=True, exist_ok=True)
        knobs = dict(plan.get("defaults", {}))
        chosen = None
        if stage.get("select_from"):
            chosen = best(root, stage["select_from"], guard)
            knobs.update(json.loads((root / chosen / "resolved.json").read_text())["knobs"])
        knobs.update(stage.get("knobs", {}))
        if "command" in stage:          # a custom command (tests, probes): knobs become its flags
            command = list(stage["command"]) + argv_for(knobs, []) + ["--output", str(folder)]
        else:
            command = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                       f"--nproc-per-node={plan.get('nproc', 8)}", "--master-addr", "127.0.0.1",
                       f"--master-port={plan.get('master_port', 29600)}", "-m", "cq_pretrain_b200.train.loop",
                       *argv_for(knobs, plan.get("common_args", [])), "--output", str(folder)]
        atomic_json(folder / "resolved.json", dict(knobs=knobs, command=command, selected_from=chosen))
        env = dict(os.environ, **{k: str(v) for k, v in stage.get("environment", {}).items()})
        with (folder / "job.log").open("w") as log:
            process = subprocess.Popen(command, env=env, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
            reason = _watch(process, folder, guard, time.monotonic() + float(stage.get("timeout_seconds", 5400)), poll)
        returncode = process.returncode if reason is None else (process.returncode or -1)
        atomic_json(folder / "exit.json", dict(returncode=returncode, rejection=reason))
        passed = returncode == 0 and reason is None
        log_text = (folder / "job.log").read_text(errors="replace").lower()
        memory_failure = not passed and (bool(reason and "memory" in reason) or "out of memory" in log_text)
        outcomes.append(dict(name=stage["name"], passed=passed, optional=stage.get("optional", False),
                             memory_failure=memory_failure, rejection=reason))
        atomic_json(root / "progress.json", dict(completed=outcomes))
        if not passed and not stage.get("optional", False):
            raise RuntimeError(f"required stage {stage['name']} failed")
        if not passed and not memory_failure:
            raise RuntimeError(f"unexpected failure in {stage['name']}; stopping the matrix for diagnosis")
    atomic_json(root / "complete.json", dict(stages=outcomes, planned_stages=len(plan["stages"]),
                                              stopped_at_boundary=(root / "stop_after_current_stage").exists()))
    return outcomes


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--plan", required=True, type=Path)
    args = parser.parse_args(argv)
    run(json.loads(args.plan.read_text()))


if __name__ == "__main__":
    main()
