"""Small host utilities: source identity, rendezvous interface, phase timer and per-rank logs."""

import json

from cq_pretrain_b200.utils import experiment, network, observe


def test_source_digest_tracks_content_and_names(tmp_path):
    (tmp_path / "pkg").mkdir()
    (tmp_path / "pkg" / "a.py").write_text("x = 1\n")
    (tmp_path / "pkg" / "k.cu").write_text("// kernel\n")
    (tmp_path / "notes.txt").write_text("ignored suffix\n")
    (tmp_path / "_build").mkdir()
    (tmp_path / "_build" / "gen.py").write_text("built = True\n")
    hashes = experiment.source_hashes(tmp_path)
    assert sorted(hashes) == ["pkg/a.py", "pkg/k.cu"]          # build output and other suffixes excluded
    first = experiment.source_digest(tmp_path)
    assert experiment.source_digest(tmp_path) == first
    (tmp_path / "pkg" / "a.py").write_text("x = 2\n")
    assert experiment.source_digest(tmp_path) != first
    (tmp_path / "pkg" / "a.py").write_text("x = 1\n")
    (tmp_path / "pkg" / "a.py").rename(tmp_path / "pkg" / "b.py")   # same bytes, new name
    assert experiment.source_digest(tmp_path) != first


def test_rendezvous_interface_for_loopback():
    name, addresses = network.rendezvous_interface("127.0.0.1")
    assert addresses[name] == "127.0.0.1"


def test_phase_timer_is_a_no_op_off_cuda():
    timer = observe.PhaseTimer("cpu")
    with observe.phase(timer, "forward"):
        pass
    with observe.phase(None, "forward"):
        pass
    assert timer.collect() == {}


def test_rank_log_rows(tmp_path):
    log = observe.RankLog(tmp_path / "out", 3)
    log.step(dict(step=1, compute_ms=12.5))
    log.acknowledged(1, [dict(serial=7, shard="s0", tensor=object(), ids=[1, 2])])
    timing = (tmp_path / "out" / "timing_rank_00003.jsonl").read_text().splitlines()
    consumed = (tmp_path / "out" / "consumed_rank_00003.jsonl").read_text().splitlines()
    assert json.loads(timing[0]) == dict(step=1, compute_ms=12.5)
    # only plain values of a receipt are logged
    assert json.loads(consumed[0]) == dict(step=1, receipts=[dict(serial=7, shard="s0", ids=[1, 2])])


def test_backend_provenance_on_a_cpu_host():
    info = observe.backend_provenance()
    for key in ("torch", "cuda_available", "kernel_library", "kernels_enabled", "native_launches",
                "tp_symmetric_workspace", "deterministic_wgrad"):
        assert key in info
    assert info["tp_symmetric_workspace"] is None          # no TP group here
    json.dumps(info)                                          # the run record stores it as JSON
