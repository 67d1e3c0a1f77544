"""The training program end to end on CPU: steps, per-rank logs, provenance, profiler traces,
checkpoint + resume through the loop (tiny configuration)."""

import json

import pytest

from cq_pretrain_b200.config import tiny_config


@pytest.mark.timeout(600)
def test_loop_writes_logs_provenance_profile_and_resumes(tmp_path):
    from cq_pretrain_b200.train import loop
    cfg = tiny_config(layers=4, dit_layers=1, vocab_size=256, width=128, ffn=256, heads=4, kv_heads=2, head_dim=32,
                      mrope_section=(2, 1, 1), linear_heads=2, linear_head_dim=32, dit_width=64, dit_heads=2,
                      dit_ffn=128)
    out = tmp_path / "run"
    rows = loop.run(cfg, tp=1, length=256, steps=3, lr=1e-4, output=out, synthetic="tiny", checkpoint_interval=2,
                    warmup_steps=1, phase_timing=True, profile=True)
    assert len(rows) == 3 and all(r["loss"] == r["loss"] for r in rows)
    timing = [json.loads(x) for x in (out / "timing_rank_00000.jsonl").read_text().splitlines()]
    consumed = [json.loads(x) for x in (out / "consumed_rank_00000.jsonl").read_text().splitlines()]
    assert [t["step"] for t in timing] == [1, 2, 3] and all(t["data_wait_seconds"] >= 0 for t in timing)
    assert [c["step"] for c in consumed] == [1, 2, 3] and consumed[0]["receipts"][0]["serial"] >= 0
    backend = json.loads((out / "backend_rank_00000.json").read_text())
    assert backend["rank"] == 0 and "kernel_library" in backend and "torch" in backend
    trace = loop._LAST_PROFILER.export(out / "profile" / "rank_00000.json")
    assert trace.exists() and trace.with_suffix(".txt").exists()
    summary = json.loads((out / "summary.json").read_text())
    assert summary["steps"] == 3
    # resume from the step-2 checkpoint through the loop: continues at step 3
    rows2 = loop.run(cfg, tp=1, length=256, steps=3, lr=1e-4, output=tmp_path / "run2", synthetic="tiny",
                     checkpoint_dir=out / "checkpoints", resume=True, warmup_steps=1)
    assert [r["step"] for r in rows2] == [3]
