"""Pinned identities of language/vision checkpoints and checks of their files.

A checkpoint directory carries ``manifest.json`` = {model_id, revision, files: {name: sha256}}.
Only the (model_id, revision) pairs in ``ALLOWED`` load (the same pins as the reference,
``utils/assets.py:20-53``: the tokenizer, vocabulary and vision geometry of these revisions are
what the token contract and the vision tower assume). ``vision_config`` accepts only the Qwen3.5
tower geometry this framework implements: patch 16, temporal patch 2, 2x2 merge, GELU-tanh MLP,
no DeepStack taps.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

ALLOWED = frozenset({
    ("Qwen/Qwen3.5-2B-Base", "b1485b2fa6dfa1287294f269f5fb618e03d52d7c"),
    ("Qwen/Qwen3.5-0.8B", "2fc06364715b967f1860aea9cf38778875588b17"),
    ("Qwen/Qwen3.5-9B", "c202236235762e1c871ad0ccb60c8ee5ba337b9a"),
    ("Qwen/Qwen3.5-9B-Base", "68c46c4b3498877f3ef123c856ecfde50c39f404"),
})


def sha256_file(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(8 << 20), b""):
            h.update(block)
    return h.hexdigest()


def asset_manifest(root, verify=False) -> dict:
    """The checkpoint's manifest; raises on an unpinned identity or (``verify``) a changed file."""
    root = Path(root)
    data = json.loads((root / "manifest.json").read_text())
    if (data.get("model_id"), data.get("revision")) not in ALLOWED:
        raise ValueError(f"checkpoint identity {data.get('model_id')}@{data.get('revision')} is not pinned")
    if verify:
        for name, digest in data.get("files", {}).items():
            if sha256_file(root / name) != digest:
                raise ValueError(f"checkpoint file changed: {name}")
    return data


def vision_config(root) -> dict:
    cfg = json.loads((Path(root) / "config.json").read_text())["vision_config"]
    if cfg.get("deepstack_visual_indexes"):
        raise ValueError("DeepStack vision towers are not supported")
    geometry = (cfg.get("patch_size"), cfg.get("temporal_patch_size"), cfg.get("spatial_merge_size"))
    if geometry != (16, 2, 2):
        raise ValueError(f"expected patch 16 / temporal 2 / merge 2, got {geometry}")
    if cfg.get("hidden_act") != "gelu_pytorch_tanh":
        raise ValueError(f"unsupported vision activation {cfg.get('hidden_act')}")
    return cfg
