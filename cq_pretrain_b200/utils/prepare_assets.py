"""Pin and verify the Qwen3.5 checkpoints this framework loads (reference ``scripts/prepare_qwen35.py``,
``scripts/prepare_qwen35_vision.py``).

``python -m cq_pretrain_b200.utils.prepare_assets pin --source DIR --output DIR --model-id ID --revision REV``
copies the files training needs (config, tokenizer and processor files, the safetensors index and
every shard it names) from a local copy of a pinned revision (``utils.assets.ALLOWED``) into
``--output`` and writes ``manifest.json`` = {model_id, revision, files: {name: sha256}, source}.
If the source carries Hugging Face repository metadata (``--upstream`` JSON, or
``.hfd/repo_metadata.json`` inside the source: ``{sha, siblings: [{rfilename, lfs: {sha256}} |
{rfilename, blobId}]}``), every copied file is also checked against the upstream hash (LFS sha256,
or the git blob sha1 of small files) and the revision must equal ``sha``. ``--vision`` also applies
the vision-tower geometry guard. ``verify --root DIR`` re-hashes a pinned directory. ``fetch``
downloads a pinned revision with ``huggingface_hub`` first (needs network access) and then pins it.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import shutil
import sys
from pathlib import Path

from .assets import ALLOWED, asset_manifest, sha256_file, vision_config

BASE_FILES = ("config.json", "tokenizer.json", "tokenizer_config.json", "preprocessor_config.json",
              "video_preprocessor_config.json", "generation_config.json", "merges.txt", "vocab.json",
              "model.safetensors.index.json", "LICENSE")


def _needed(source: Path):
    names = [n for n in BASE_FILES if (source / n).is_file()]
    index = source / "model.safetensors.index.json"
    if index.is_file():
        names += sorted(set(json.loads(index.read_text())["weight_map"].values()))
    elif (source / "model.safetensors").is_file():
        names.append("model.safetensors")
    if "config.json" not in names:
        raise ValueError(f"{source} has no config.json: not a checkpoint directory")
    return names


def _git_blob_sha1(path: Path):
    h = hashlib.sha1()
    h.update(f"blob {path.stat().st_size}\0".encode())
    with path.open("rb") as handle:
        for block in iter(lambda: handle.read(8 << 20), b""):
            h.update(block)
    return h.hexdigest()


def check_upstream(root: Path, metadata: dict, revision: str, names):
    """Compare every file in ``names`` that the upstream listing knows with its upstream hash."""
    if metadata.get("sha") != revision:
        raise ValueError(f"upstream metadata is for revision {metadata.get('sha')}, not {revision}")
    listing = {item["rfilename"]: item for item in metadata.get("siblings", [])}
    for name in names:
        item = listing.get(name)
        if item is None:
            continue
        if "lfs" in item:
            ok = sha256_file(root / name) == item["lfs"]["sha256"]
        else:
            ok = _git_blob_sha1(root / name) == item.get("blobId")
        if not ok:
            raise ValueError(f"{name} does not match the upstream repository hash")


def pin(source, output, model_id, revision, upstream=None, vision=False):
    source, output = Path(source).resolve(), Path(output).resolve()
    if (model_id, revision) not in ALLOWED:
        raise ValueError(f"{model_id}@{revision} is not a pinned checkpoint identity")
    output.mkdir(parents=True, exist_ok=True)
    if (output / "manifest.json").exists():
        raise FileExistsError(f"{output} is already pinned; use verify")
    names = _needed(source)
    files = {}
    for name in names:
        target = output / name
        target.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(source / name, target)
        files[name] = sha256_file(target)
    metadata = None
    if upstream is not None:
        metadata = json.loads(Path(upstream).read_text())
    elif (source / ".hfd" / "repo_metadata.json").is_file():
        metadata = json.loads((source / ".hfd" / "repo_metadata.json").read_text())
    if metadata is not None:
        check_upstream(output, metadata, revision, names)
    if vision:
        vision_config(output)
    manifest = dict(model_id=model_id, revision=revision, files=files, source=str(source),
                    upstream_checked=metadata is not None)
    (output / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def verify(root, vision=False):
    manifest = asset_manifest(root, verify=True)
    if vision:
        vision_config(root)
    return manifest


def fetch(model_id, revision, output, vision=False):
    try:
        from huggingface_hub import snapshot_download
    except ImportError as error:
        raise RuntimeError("fetch needs huggingface_hub; pin a local copy with `pin --source` instead") from error
    if (model_id, revision) not in ALLOWED:
        raise ValueError(f"{model_id}@{revision} is not a pinned checkpoint identity")
    staging = Path(output).resolve().with_name(Path(output).name + ".download")
    snapshot_download(repo_id=model_id, revision=revision, local_dir=str(staging))
    return pin(staging, output, model_id, revision, vision=vision)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = parser.add_subparsers(dest="command", required=True)
    p = sub.add_parser("pin")
    p.add_argument("--source", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--model-id", required=True)
    p.add_argument("--revision", required=True)
    p.add_argument("--upstream", default=None)
    p.add_argument("--vision", action="store_true")
    v = sub.add_parser("verify")
    v.add_argument("--root", required=True)
    v.add_argument("--vision", action="store_true")
    f = sub.add_parser("fetch")
    f.add_argument("--model-id", required=True)
    f.add_argument("--revision", required=True)
    f.add_argument("--output", required=True)
    f.add_argument("--vision", action="store_true")
    args = parser.parse_args(argv)
    if args.command == "pin":
        out = pin(args.source, args.output, args.model_id, args.revision, args.upstream, args.vision)
    elif args.command == "verify":
        out = verify(args.root, args.vision)
    else:
        out = fetch(args.model_id, args.revision, args.output, args.vision)
    print(json.dumps(dict(status=args.command, model_id=out["model_id"], revision=out["revision"],
                          files=len(out["files"]))), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
