"""Launch generation protocol, launcher dry run, corpus stream resumption (CPU)."""

import json
import sys
import threading
from pathlib import Path

import numpy as np
import pytest

from cq_pretrain_b200.data.stream import DocumentStream, permute
from cq_pretrain_b200.launch import launcher, supervisor


def test_two_nodes_agree_on_one_generation(tmp_path):
    results = {}

    def node(rank):
        results[rank] = supervisor.join_attempt(tmp_path, rank, 2, timeout=30, interval=0.05)

    threads = [threading.Thread(target=node, args=(r,)) for r in (1, 0)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert results[0] == results[1]
    sealed = json.loads((tmp_path / "generations" / results[0] / "sealed.json").read_text())
    assert len(sealed["members"]) == 2


def test_second_registration_of_a_node_is_refused(tmp_path):
    (tmp_path / "LATEST").write_text(json.dumps(dict(generation="g", nodes=2)))
    (tmp_path / "generations" / "g" / "members").mkdir(parents=True)
    (tmp_path / "generations" / "g" / "members" / "001.json").write_text(json.dumps(dict(token="other")))
    with pytest.raises(RuntimeError, match="already registered"):
        supervisor.join_attempt(tmp_path, 1, 2, timeout=5, interval=0.05)


def test_topology_change_is_rejected(tmp_path):
    (tmp_path / "LATEST").write_text(json.dumps(dict(generation="g", nodes=3)))
    with pytest.raises(ValueError):
        supervisor.join_attempt(tmp_path, 1, 2, timeout=5, interval=0.05)


def test_peer_failure_stops_the_local_child(tmp_path):
    attempt = tmp_path / "attempt"
    attempt.mkdir()
    (tmp_path / "LATEST").write_text(json.dumps(dict(generation="g", nodes=2)))
    (attempt / "exit_node_001.json").write_text(json.dumps(dict(exit_code=1)))
    code = supervisor.supervise([sys.executable, "-c", "import time; time.sleep(60)"], attempt, tmp_path, "g", 0, 2,
                                poll=0.05, grace=5)
    assert code != 0
    assert json.loads((attempt / "exit_node_000.json").read_text())["exit_code"] == code


def test_clean_exit_marks_complete(tmp_path):
    attempt = tmp_path / "attempt"
    attempt.mkdir()
    (tmp_path / "LATEST").write_text(json.dumps(dict(generation="g", nodes=1)))
    code = supervisor.supervise([sys.executable, "-c", "pass"], attempt, tmp_path, "g", 0, 1, poll=0.05)
    assert code == 0
    assert supervisor.finish(tmp_path, attempt, "g", 0, 1, timeout=5) == 0
    assert json.loads((tmp_path / "complete.json").read_text())["status"] == "finite_dataset_complete"


def test_launcher_dry_run(capsys, tmp_path):
    launcher.main(["--rendezvous", str(tmp_path / "r"), "--nodes", "1", "--node-rank", "0", "--nproc-per-node", "8",
                   "--dry-run", "--", "--config", "x.yaml"])
    out = json.loads(capsys.readouterr().out)
    assert out["world"] == 8 and "--nproc-per-node=8" in out["command"]


def test_feistel_is_a_permutation():
    for n in (1, 7, 64, 1000):
        values = [permute(i, n, seed=3, epoch=1) for i in range(n)]
        assert sorted(values) == list(range(n))
    assert [permute(i, 100, 3, 0) for i in range(100)] != [permute(i, 100, 3, 1) for i in range(100)]


def _corpus(root, n=40):
    root.mkdir()
    with (root / "docs.jsonl").open("w") as f:
        for i in range(n):
            f.write(json.dumps(dict(id=f"d{i}", elements=[dict(type="text", input_ids=[i + 10] * (i % 5 + 1))])) + "\n")


def test_stream_shards_and_resumes(tmp_path):
    _corpus(tmp_path / "c")
    seen = []
    for rank in range(2):
        s = DocumentStream(tmp_path / "c", seed=1, rank=rank, world=2, block_rows=4)
        while (d := s.peek()) is not None:
            seen.append(d["id"])
            s.advance()
    assert sorted(seen) == sorted(f"d{i}" for i in range(40))   # every document exactly once
    a = DocumentStream(tmp_path / "c", seed=1, rank=0, world=2)
    for _ in range(5):
        a.peek()
        a.advance()
    state = a.state_dict()
    rest_a = []
    while (d := a.peek()) is not None:
        rest_a.append(d["id"])
        a.advance()
    b = DocumentStream(tmp_path / "c", seed=1, rank=0, world=2)
    b.load_state_dict(state)
    rest_b = []
    while (d := b.peek()) is not None:
        rest_b.append(d["id"])
        b.advance()
    assert rest_a == rest_b
    with pytest.raises(ValueError):
        DocumentStream(tmp_path / "c", seed=2, rank=0, world=2).load_state_dict(state)


def test_committed_yaml_configs_load_and_validate():
    from pathlib import Path
    from cq_pretrain_b200.config import load_sections, tiny_config
    root = Path(__file__).resolve().parents[1] / "cq_pretrain_b200" / "configs"
    cfg, training, env = load_sections(root / "qwen35_2b_wan.yaml")
    cfg.validate(int(training["tp"]))
    assert cfg.width == 2048 and training["sequence_length"] == 8192 and "PYTORCH_CUDA_ALLOC_CONF" in env
    tiny, _, _ = load_sections(root / "tiny.yaml")
    assert tiny.to_dict() == tiny_config().to_dict()


def test_launcher_receipts_must_agree(tmp_path):
    mine = launcher.Receipt("a", "10.0.0.1", "eth0", {"x.py": "1", "y.py": "2"}, 8)
    other = launcher.Receipt("b", "10.0.0.2", "eth0", {"x.py": "1", "y.py": "3"}, 4)
    problems = launcher.disagreements([mine, other], mine)
    assert len(problems) == 2 and "y.py" in problems[1] and "4 processes" in problems[0]
    r = launcher.Rendezvous(tmp_path / "r", 2, 0)
    r.publish(mine)
    with pytest.raises(FileExistsError):
        r.publish(mine)
    launcher.Rendezvous(tmp_path / "r", 2, 1).publish(other)
    assert [x.hostname for x in r.collect(timeout=5)] == ["a", "b"]
    env = launcher.launch_environment({"RANK": "3", "PATH": "/bin"}, "10.0.0.1", 29500, "eth0")
    assert "RANK" not in env and env["NCCL_SOCKET_IFNAME"] == "eth0" and env["MASTER_ADDR"] == "10.0.0.1"
