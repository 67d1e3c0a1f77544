"""Corpus sources (Parquet row-group index, JSONL task records, YAML mixtures) and the threaded
document stream with tokenization and visual loading ahead of the cursor (CPU)."""

import hashlib
import json
import threading

import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from cq_pretrain_b200.data.catalog import JsonlSource, MixedSource, ParquetSource, normalize_task_record
from cq_pretrain_b200.data.stream import DocumentStream


def _parquet_corpus(root, files=3, rows=10, group=4, manifest=True):
    root.mkdir(parents=True)
    entries = []
    for f in range(files):
        docs = [dict(id=f"f{f}r{r}", elements=json.dumps([dict(type="text", input_ids=[f * 100 + r + 10] * 3)]))
                for r in range(rows)]
        path = root / f"part{f}.parquet"
        pq.write_table(pa.Table.from_pylist(docs), path, row_group_size=group)
        entries.append(dict(path=path.name, rows=rows, sha256=hashlib.sha256(path.read_bytes()).hexdigest()))
    if manifest:
        (root / "manifest.json").write_text(json.dumps(dict(snapshot="snap1", files=entries)))
        (root / "COMPLETE").write_text("")
    return root


def test_parquet_source_indexes_row_groups_and_bounds_its_cache(tmp_path):
    src = ParquetSource(_parquet_corpus(tmp_path / "c"), cache_bytes=1)
    assert len(src) == 30 and len(src.groups) == 9          # 3 files x ceil(10 / 4) row groups
    assert src.read(13)["id"] == "f1r3" and src.read(29)["id"] == "f2r9"
    assert src.read(0)["elements"][0]["input_ids"] == [10, 10, 10]
    assert len(src._cache) == 1                              # the cache keeps within its budget
    with pytest.raises(IndexError):
        src.read(30)


def test_parquet_source_checks_completeness_and_content(tmp_path):
    root = _parquet_corpus(tmp_path / "c")
    (root / "COMPLETE").unlink()
    with pytest.raises(ValueError, match="COMPLETE"):
        ParquetSource(root)
    (root / "COMPLETE").write_text("")
    src = ParquetSource(root)
    # rewrite one file with the same row count: caught when its rows are first read
    pq.write_table(pa.Table.from_pylist([dict(id=f"x{r}", elements="[]") for r in range(10)]), root / "part2.parquet",
                   row_group_size=4)
    assert src.read(3)["id"] == "f0r3"
    with pytest.raises(ValueError, match="changed"):
        src.read(25)


def test_task_records_normalise_into_conversations(tmp_path):
    (tmp_path / "a.jpg").write_bytes(b"x")
    rows = [dict(task="t2i", caption="a red cube", image_path="a.jpg"),
            dict(task="i2t", caption="a blue ball", image_path="a.jpg", sample_id="s2"),
            dict(task="v2t", caption="a dog runs", video_path="a.mp4", fps=2),
            dict(task="t2i", messages=[dict(role="user", content=[dict(type="image")]),
                                       dict(role="assistant", content="no")], images=[dict(path="a.jpg")])]
    path = tmp_path / "t.jsonl"
    path.write_text("\n".join(json.dumps(r) for r in rows) + "\n\n")
    src = JsonlSource(path)
    assert len(src) == 4
    t2i = src.read(0)
    assert t2i["direction"] == "T2I" and [s["kind"] for s in t2i["segments"]] == ["text", "image"]
    assert t2i["segments"][1]["role"] == "assistant" and t2i["images"][0]["path"].endswith("a.jpg")
    i2t = src.read(1)
    assert i2t["sample_id"] == "s2" and i2t["segments"][0]["kind"] == "image" and not i2t["image_loss_allowed"]
    v2t = src.read(2)
    assert v2t["images"][0]["video"] and v2t["images"][0]["fps"] == 2
    with pytest.raises(ValueError, match="assistant"):
        src.read(3)
    with pytest.raises(ValueError, match="task"):
        normalize_task_record(dict(caption="x"), {}, path, 0)


def test_yaml_mixture_concatenates_sources(tmp_path):
    _parquet_corpus(tmp_path / "pq", files=1, rows=5, manifest=False)
    (tmp_path / "t.jsonl").write_text(json.dumps(dict(caption="hello", image_path="z.jpg")) + "\n")
    (tmp_path / "mix.yaml").write_text("sources:\n  - path: pq\n  - path: t.jsonl\n    task: t2i\n")
    mix = MixedSource(tmp_path / "mix.yaml")
    assert len(mix) == 6
    assert mix.read(4)["sample_id"] == "0:f0r4" and mix.read(5)["direction"] == "T2I"
    assert mix.read(5)["sample_id"].startswith("1:")


def test_stream_tokenizes_ahead_in_threads_and_resumes_exactly(tmp_path):
    rows = [dict(sample_id=f"d{i}", format="natural", segments=[dict(kind="text", text="ab" * (i % 5 + 1))])
            for i in range(40)]
    (tmp_path / "raw.jsonl").write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    threads = set()

    def encode(text):
        threads.add(threading.current_thread().name)
        return [ord(c) for c in text]

    s = DocumentStream(tmp_path / "raw.jsonl", seed=4, rank=0, world=2, block_rows=4, encode=encode, workers=3,
                       lookahead=8)
    seen = []
    for _ in range(6):
        doc = s.peek()
        seen.append((doc["id"], list(doc["elements"][0]["input_ids"])))
        s.advance()
    assert any(name.startswith("docstream") for name in threads)     # prepared by the pool
    state = s.state_dict()
    rest = []
    while (doc := s.peek()) is not None:
        rest.append(doc["id"])
        s.advance()
    s.close()
    assert len(seen) + len(rest) == 20                              # rank 0 gets half of the blocks
    resumed = DocumentStream(tmp_path / "raw.jsonl", seed=4, rank=0, world=2, block_rows=4, encode=encode,
                             workers=0)
    resumed.load_state_dict(state)
    again = []
    while (doc := resumed.peek()) is not None:
        again.append(doc["id"])
        resumed.advance()
    assert again == rest
    assert all(ids == [ord(c) for c in "ab" * (int(i[1:]) % 5 + 1)] for i, ids in seen)
