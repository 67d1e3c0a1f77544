"""Corpus sources that index their rows without loading them (reference ``data/catalog.py:19-155``,
``data/sources.py:11-132``).

* ``ParquetSource``: a directory of Parquet files (``manifest.json`` + ``COMPLETE`` when the
  snapshot is published). Construction reads only file metadata: each file's row groups become
  index entries, so locating row ``i`` is a binary search. Reading a row decodes its whole row
  group into a bounded LRU cache (``cache_bytes``). A file listed in the manifest is hashed
  (streaming sha256) the first time one of its rows is read, and must match the manifest.
* ``JsonlSource``: one JSONL file, indexed by the byte offset of every non-empty line (one
  streaming pass); a row is one ``seek`` + ``readline``. Task records (``task`` t2i / i2t / t2v /
  v2t with a caption, or chat ``messages``) are normalised into the corpus row format
  (``segments``, ``images``, ``format``, ``direction``) by ``normalize_task_record``.
* ``MixedSource``: a YAML file ``sources: [{path: ..., task: ..., caption_field: ..., ...}]``
  concatenating Parquet directories and JSONL files (sample ids prefixed by the source index).

Every source has ``len()``, ``read(i)`` (a row dict), ``identity`` (a digest that changes when
the data does; resumed streams compare it) and ``close()``.
"""

from __future__ import annotations

import hashlib
import json
import threading
from array import array
from bisect import bisect_right
from collections import OrderedDict
from pathlib import Path


def digest(value):
    return hashlib.sha256(json.dumps(value, sort_keys=True).encode()).hexdigest()[:32]


def _file_sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(1 << 22), b""):
            h.update(block)
    return h.hexdigest()


class ParquetSource:
    def __init__(self, root, cache_bytes=256 << 20):
        import pyarrow.parquet as pq
        self.root = Path(root)
        manifest = self.root / "manifest.json"
        self.manifest = json.loads(manifest.read_text()) if manifest.exists() else None
        if self.manifest is not None:
            if not (self.root / "COMPLETE").exists():
                raise ValueError(f"corpus snapshot {self.root} is not COMPLETE")
            entries = self.manifest["files"]
            files = [self.root / e["path"] for e in entries]
            self.expected = {str(self.root / e["path"]): e for e in entries}
        else:
            files = sorted(self.root.glob("*.parquet"))
            self.expected = {}
        self.files, self.groups, self.ends = [], [], []    # (file index, row group) per index entry
        total = 0
        for fi, path in enumerate(files):
            meta = pq.ParquetFile(path).metadata
            want = self.expected.get(str(path), {}).get("rows")
            if want is not None and want != meta.num_rows:
                raise ValueError(f"{path} holds {meta.num_rows} rows, the manifest says {want}")
            self.files.append(path)
            for g in range(meta.num_row_groups):
                total += meta.row_group(g).num_rows
                self.groups.append((fi, g))
                self.ends.append(total)
        self.rows = total
        self.snapshot = self.manifest.get("snapshot", "unversioned") if self.manifest else "unversioned"
        self.identity = digest(dict(snapshot=self.snapshot, files=[str(p.name) for p in self.files], rows=total))
        self.cache_bytes = cache_bytes
        self._cache = OrderedDict()        # entry -> (rows, bytes)
        self._cached_bytes = 0
        self._verified = set()
        self._lock = threading.Lock()
        self._handles = {}

    def __len__(self):
        return self.rows

    def _verify(self, fi):
        path = self.files[fi]
        entry = self.expected.get(str(path))
        if entry and "sha256" in entry and _file_sha256(path) != entry["sha256"]:
            raise ValueError(f"corpus file changed since publication: {path}")
        self._verified.add(fi)

    def _group_rows(self, entry):
        with self._lock:
            hit = self._cache.get(entry)
            if hit is not None:
                self._cache.move_to_end(entry)
                return hit[0]
        import pyarrow.parquet as pq
        fi, g = self.groups[entry]
        if fi not in self._verified:
            self._verify(fi)
        table = pq.ParquetFile(self.files[fi]).read_row_group(g)
        rows, size = table.to_pylist(), table.nbytes
        with self._lock:
            self._cache[entry] = (rows, size)
            self._cached_bytes += size
            while self._cached_bytes > self.cache_bytes and len(self._cache) > 1:
                _, (_, dropped) = self._cache.popitem(last=False)
                self._cached_bytes -= dropped
        return rows

    def read(self, index):
        if not 0 <= index < self.rows:
            raise IndexError(index)
        entry = bisect_right(self.ends, index)
        first = self.ends[entry - 1] if entry else 0
        row = dict(self._group_rows(entry)[index - first])
        for key in ("elements", "segments", "images", "messages"):
            if isinstance(row.get(key), str):
                row[key] = json.loads(row[key])
        return row

    def close(self):
        self._cache.clear()


def normalize_task_record(row, source, path, index):
    """A task-style JSONL record -> the corpus row format the chat templating reads.

    ``task`` (record or source default) is t2i / i2t / t2v / v2t. Visuals come from ``images`` /
    ``videos`` lists or a single ``image_path`` / ``video_path`` (relative paths resolve against
    the JSONL's directory). Without ``messages`` the record's caption (``caption_field``, default
    ``caption``) forms a user turn and the visual the assistant turn for generation tasks, the
    other way round for understanding tasks. Generation targets must sit in assistant turns and
    understanding visuals in user turns.
    """
    task = str(row.get("task", source.get("task", ""))).lower()
    if task not in ("t2i", "i2t", "t2v", "v2t"):
        raise ValueError(f"{path}:{index}: a task record needs task t2i, i2t, t2v or v2t")
    video = "v" in task
    generate = task.startswith("t")
    media = row.get("videos" if video else "images")
    if media is None:
        single = dict(path=row.get("video_path" if video else "image_path"))
        single.update({k: row[k] for k in ("frames_path", "fps", "start_seconds", "num_frames") if k in row})
        media = [single]
    media = [dict(m) for m in media]
    for item in media:
        for key in ("path", "frames_path"):
            if item.get(key):
                item[key] = str((Path(path).parent / item[key]).resolve())
        if video:
            item["video"] = True
            item["settings"] = source.get("video", {"mode": "native"})
    messages = row.get("messages")
    if messages is None:
        caption = dict(type="text", text=row[source.get("caption_field", "caption")])
        visual = dict(type="video" if video else "image", index=0)
        first, second = (caption, visual) if generate else (visual, caption)
        messages = [dict(role="user", content=[first]), dict(role="assistant", content=[second])]
    segments, visual_roles = [], []
    for turn, message in enumerate(messages):
        content = message["content"]
        if isinstance(content, str):
            content = [dict(type="text", text=content)]
        for item in content:
            seg = dict(role=message["role"], turn=turn)
            if item["type"] == "text":
                seg.update(kind="text", text=item["text"])
            elif item["type"] in ("image", "video"):
                slot = item.get("index", 0)
                if "video_id" in item:
                    slot = next(i for i, m in enumerate(media) if m.get("id", "v0") == item["video_id"])
                if not 0 <= slot < len(media):
                    raise ValueError(f"{path}:{index}: visual reference {slot} out of range")
                seg.update(kind="image", image_index=slot)
                visual_roles.append(message["role"])
            else:
                raise ValueError(f"{path}:{index}: unsupported content type {item['type']!r}")
            segments.append(seg)
    wanted = "assistant" if generate else "user"
    if not visual_roles or any(role != wanted for role in visual_roles):
        raise ValueError(f"{path}:{index}: {'generation targets' if generate else 'understanding visuals'} "
                         f"belong in {wanted} turns")
    return dict(row, sample_id=str(row.get("sample_id", f"{Path(path).stem}:{index}")), images=media,
                segments=segments, format="conversation", direction=task.upper(),
                image_loss_allowed=generate and row.get("image_loss_allowed", True))


class JsonlSource:
    def __init__(self, path, source=None):
        self.path = Path(path).resolve()
        self.source = dict(source or {})
        self.offsets = array("Q")
        h = hashlib.sha256()
        with self.path.open("rb") as handle:
            position = 0
            for line in handle:
                h.update(line)
                if line.strip():
                    self.offsets.append(position)
                position += len(line)
        self.identity = digest(dict(sha256=h.hexdigest(), source=self.source))
        self.snapshot = f"jsonl:{self.identity}"
        self._local = threading.local()

    def __len__(self):
        return len(self.offsets)

    def read(self, index):
        handle = getattr(self._local, "handle", None)
        if handle is None:
            handle = self._local.handle = self.path.open("rb")
        handle.seek(self.offsets[index])
        row = json.loads(handle.readline())
        if "elements" in row or "segments" in row:
            return row
        return normalize_task_record(row, self.source, self.path, index)

    def close(self):
        handle = getattr(self._local, "handle", None)
        if handle is not None:
            handle.close()
            self._local.handle = None


class MixedSource:
    """``spec``: a YAML file path, or a list of ``{path, ...options}`` (paths relative to ``base``)."""

    def __init__(self, spec, cache_bytes=256 << 20, base=None):
        if isinstance(spec, (str, Path)):
            import yaml
            self.path = Path(spec).resolve()
            items, base = yaml.safe_load(self.path.read_text())["sources"], self.path.parent
        else:
            self.path, items = None, list(spec)
            base = Path(base or ".")
        self.sources, self.ends, total = [], [], 0
        for item in items:
            target = (Path(base) / item["path"]).resolve()
            options = {k: v for k, v in item.items() if k != "path"}
            source = ParquetSource(target, cache_bytes) if target.is_dir() else JsonlSource(target, options)
            self.sources.append(source)
            total += len(source)
            self.ends.append(total)
        self.rows = total
        self.identity = digest([s.identity for s in self.sources])
        self.snapshot = f"mixed:{self.identity}"

    def __len__(self):
        return self.rows

    def read(self, index):
        which = bisect_right(self.ends, index)
        first = self.ends[which - 1] if which else 0
        row = self.sources[which].read(index - first)
        row["sample_id"] = f"{which}:{row.get('sample_id', row.get('id', index - first))}"
        return row

    def close(self):
        for s in self.sources:
            s.close()


def open_source(path, cache_bytes=256 << 20):
    """A Parquet directory, a JSONL file, or a YAML mixture of both."""
    path = Path(path)
    if path.is_dir():
        jsonl = sorted(path.glob("*.jsonl"))
        if jsonl and not any(path.glob("*.parquet")) and not (path / "manifest.json").exists():
            if len(jsonl) == 1:
                return JsonlSource(jsonl[0])
            return MixedSource([dict(path=p.name) for p in jsonl], cache_bytes, base=path)
        return ParquetSource(path, cache_bytes)
    if path.suffix == ".jsonl":
        return JsonlSource(path)
    return MixedSource(path, cache_bytes)
