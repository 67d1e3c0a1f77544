"""Staged tuning matrix: selection by throughput under a memory guard, kills, skips (CPU, fake jobs)."""

import json
import sys
import textwrap

import pytest

from cq_pretrain_b200.launch.tune import run

JOB = textwrap.dedent("""
    import json, sys, time
    from pathlib import Path
    args = sys.argv[1:]
    out = Path(args[args.index('--output') + 1])
    opts = {args[i][2:]: args[i + 1] for i in range(len(args) - 1) if args[i].startswith('--')}
    rate, peak = float(opts.get('rate', 1)), float(opts.get('peak', 1))
    if opts.get('mode') == 'fail':
        sys.exit(3)
    with (out / 'steps.jsonl').open('a') as f:
        f.write(json.dumps(dict(step=1, peak_gib=peak)) + '\\n')
    if opts.get('mode') == 'hang':
        time.sleep(60)
    (out / 'summary.json').write_text(json.dumps(dict(content_tokens_per_second=rate, peak_gib=peak)))
""")


def test_matrix_selection_guard_and_skips(tmp_path):
    job = tmp_path / "job.py"
    job.write_text(JOB)
    cmd = [sys.executable, str(job)]
    plan = dict(output=str(tmp_path / "out"), memory_guard_gib=10, defaults=dict(rate=1), stages=[
        dict(name="a", command=cmd, knobs=dict(rate=5, peak=4)),
        dict(name="b", command=cmd, knobs=dict(rate=9, peak=8)),
        dict(name="big", command=cmd, knobs=dict(rate=99, peak=50), optional=True),      # stopped by the guard
        dict(name="pick", command=cmd, select_from=["a", "b", "big"], knobs=dict(extra=1)),
        dict(name="needs", command=cmd, requires_success=["big"]),
    ])
    outcomes = run(plan, poll=0.2)
    by = {o["name"]: o for o in outcomes}
    assert by["a"]["passed"] and by["b"]["passed"]
    assert not by["big"]["passed"] and by["big"]["memory_failure"]
    resolved = json.loads((tmp_path / "out" / "pick" / "resolved.json").read_text())
    assert resolved["selected_from"] == "b" and resolved["knobs"]["rate"] == 9 and resolved["knobs"]["extra"] == 1
    assert by["needs"]["skipped"]


def test_required_failure_stops(tmp_path):
    job = tmp_path / "job.py"
    job.write_text(JOB)
    plan = dict(output=str(tmp_path / "out"), stages=[
        dict(name="x", command=[sys.executable, str(job)], knobs=dict(mode="fail"))])
    with pytest.raises(RuntimeError, match="required stage x failed"):
        run(plan, poll=0.2)


def test_deadline_kills_and_stops(tmp_path):
    job = tmp_path / "job.py"
    job.write_text(JOB)
    plan = dict(output=str(tmp_path / "out"), stages=[
        dict(name="slow", command=[sys.executable, str(job)], knobs=dict(mode="hang"), optional=True,
             timeout_seconds=2)])
    with pytest.raises(RuntimeError, match="unexpected failure in slow"):
        run(plan, poll=0.2)
    progress = json.loads((tmp_path / "out" / "progress.json").read_text())
    assert progress["completed"][0]["rejection"] == dict(deadline=True)
