"""Immutable, content-addressed caches of visual features (Qwen merger) and Wan latents.

An entry's identity is a JSON dict: schema, source (e.g. the image's sha256), clip geometry,
encoder identity (sha256 over the encoder's weight and config files or its manifest) and the
preprocessing parameters. The file lives at ``root/<key[:2]>/<key>.pt`` with
``key = sha256(canonical JSON of the identity)`` and stores the identity, the tensors and a
sha256 of every tensor's bytes. ``save`` writes a temp file, fsyncs it and publishes it with
``os.link`` (first writer wins; concurrent writers of one identity are safe); ``load`` rejects a
file whose identity or checksums differ (reference ``data/cache.py:11-79``).
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
from functools import lru_cache
from pathlib import Path

import torch

SCHEMA = "cq.visual.v1"


def canonical_digest(value) -> str:
    text = json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False)
    return hashlib.sha256(text.encode()).hexdigest()


def tensor_digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _file_digest(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


@lru_cache(maxsize=16)
def encoder_identity(root) -> str:
    """Identity of an encoder checkpoint directory (or single file).

    With a ``manifest.json`` (model id, revision, file hashes) the manifest fields define it;
    otherwise the hashes of the weight files and config JSONs do.
    """
    root = Path(root)
    manifest = root / "manifest.json"
    if manifest.is_file():
        value = json.loads(manifest.read_text())
        return canonical_digest({k: value[k] for k in ("model_id", "revision", "files")})
    if root.is_file():
        names = [root]
    else:
        weights = sorted(root.glob("*.safetensors")) or sorted(root.glob("*.pth")) or sorted(root.glob("*.pt"))
        names = weights + sorted(root.glob("*config*.json"))
    return canonical_digest([(p.name, _file_digest(p)) for p in names])


class VisualCache:
    def __init__(self, root, encoder: str, preprocessing: dict):
        self.root, self.encoder, self.preprocessing = Path(root), encoder, dict(preprocessing)

    def identity(self, source, clip=None) -> dict:
        return dict(schema=SCHEMA, source=source, clip=clip, encoder=self.encoder, preprocessing=self.preprocessing)

    def path(self, identity) -> Path:
        key = canonical_digest(identity)
        return self.root / key[:2] / f"{key}.pt"

    def load(self, identity):
        path = self.path(identity)
        if not path.exists():
            return None
        payload = torch.load(path, map_location="cpu", weights_only=True)
        if payload["identity"] != identity:
            raise ValueError(f"visual cache identity differs: {path}")
        tensors = payload["tensors"]
        if payload["sha256"] != {k: tensor_digest(v) for k, v in tensors.items()}:
            raise ValueError(f"visual cache checksum differs: {path}")
        return tensors

    def save(self, identity, **tensors) -> Path:
        path = self.path(identity)
        if self.load(identity) is not None:
            return path
        path.parent.mkdir(parents=True, exist_ok=True)
        tensors = {k: v.detach().cpu().contiguous() for k, v in tensors.items()}
        payload = dict(identity=identity, tensors=tensors, sha256={k: tensor_digest(v) for k, v in tensors.items()})
        fd, tmp = tempfile.mkstemp(dir=path.parent, prefix="." + path.name)
        try:
            with os.fdopen(fd, "wb") as out:
                torch.save(payload, out)
                out.flush()
                os.fsync(out.fileno())
            try:
                os.link(tmp, path)
            except FileExistsError:
                pass
        finally:
            Path(tmp).unlink(missing_ok=True)
        self.load(identity)   # verify what was published
        return path


def caches(cfg):
    """``(qwen, wan)`` caches of a run config, or ``(None, None)`` without ``cfg.visual_cache``.

    Cached merger features are only valid for a frozen tower and merger of the backbone width.
    """
    if not getattr(cfg, "visual_cache", None):
        return None, None
    if not (cfg.freeze_vision and cfg.freeze_vision_merger):
        raise ValueError("visual caches require a frozen vision tower and merger")
    common = dict(version="native-qwen-wan-v1")
    vision = getattr(cfg, "vision_assets", None)
    vae = getattr(cfg, "wan_vae_assets", None)
    qwen = VisualCache(Path(cfg.visual_cache) / "qwen", encoder_identity(vision) if vision else "synthetic",
                       dict(common, min_pixels=cfg.vision_min_pixels, max_pixels=cfg.vision_max_pixels))
    wan = VisualCache(Path(cfg.visual_cache) / "wan", encoder_identity(vae) if vae else "synthetic",
                      dict(common, max_pixels=cfg.generation_max_pixels, posterior="mode", spatial_stride=8,
                           temporal_stride=4))
    return qwen, wan


def attach_cached(element, qwen, wan):
    """Fill ``features`` / ``latent`` (+ ``latent_shape``) of an image element from the caches by its
    ``source`` identity. A missing feature entry is an error (the tower is frozen, so training
    must not silently recompute it); a missing latent only drops the generation target."""
    if element.get("type") != "image" or "source" not in element:
        return element
    clip = element.get("clip")
    if qwen is not None and element.get("features") is None:
        found = qwen.load(qwen.identity(element["source"], clip))
        if found is None:
            raise KeyError(f"no cached merger features for {element['source']}")
        element["features"] = found["features"]
    if wan is not None and element.get("latent") is None:
        found = wan.load(wan.identity(element["source"], clip))
        if found is not None:
            element["latent"] = found["latent"]
            element["latent_shape"] = tuple(found["latent"].shape)
        else:
            element["generation_target"] = False
    return element
