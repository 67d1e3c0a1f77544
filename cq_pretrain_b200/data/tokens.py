"""Token contract between the packer, the model config and the language checkpoint's tokenizer.

The special ids are read from the tokenizer's ``tokenizer_config.json`` (``added_tokens_decoder``),
never from corpus statistics (reference ``data/packing.py:33-44``, ``data/tokenizer.py:6-28``):

=========  =====================  ======================================
role       token                  use
=========  =====================  ======================================
bos        ``<|im_start|>``       document opener (chat documents)
eos        ``<|endoftext|>``      document end
boi / eoi  ``<|vision_start|>`` / ``<|vision_end|>``  brackets of a visual element
image      ``<|image_pad|>``      visual content slot; also the visual query mask id
text_mask  ``<|fim_pad|>``        text query mask id
=========  =====================  ======================================

``token_contract`` also sets ``cfg.text_mask_token_id`` / ``cfg.image_mask_token_id`` and refuses a
tokenizer whose ids the model vocabulary cannot represent. ``tokenizer_metadata`` records the
sha256 of the tokenizer files so a resumed run can prove it tokenizes the same way.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

REQUIRED = {"bos": "<|im_start|>", "eos": "<|endoftext|>", "boi": "<|vision_start|>",
            "eoi": "<|vision_end|>", "image": "<|image_pad|>", "text_mask": "<|fim_pad|>"}
TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json")


def added_tokens(root):
    config = json.loads((Path(root) / "tokenizer_config.json").read_text())
    return {entry["content"]: int(key) for key, entry in config["added_tokens_decoder"].items()}


def special_token_ids(root):
    """Ids flagged ``special`` (excluded when counting corpus tokens)."""
    config = json.loads((Path(root) / "tokenizer_config.json").read_text())
    return sorted(int(k) for k, v in config["added_tokens_decoder"].items() if v.get("special", False))


def token_contract(root, cfg):
    """Map roles to ids from the tokenizer at ``root`` and set the config's mask ids."""
    added = added_tokens(root)
    missing = [text for text in REQUIRED.values() if text not in added]
    if missing:
        raise ValueError(f"tokenizer lacks required special tokens: {missing}")
    tokens = {role: added[text] for role, text in REQUIRED.items()}
    if max(tokens.values()) >= cfg.vocab_size:
        raise ValueError("model vocabulary cannot represent the tokenizer's special ids")
    cfg.text_mask_token_id = tokens["text_mask"]
    cfg.image_mask_token_id = tokens["image"]
    return tokens


def synthetic_contract(cfg):
    """Token ids for synthetic runs without a tokenizer: the first ids of the vocabulary."""
    tokens = dict(bos=0, eos=1, boi=2, eoi=3, image=cfg.image_mask_token_id, text_mask=cfg.text_mask_token_id)
    if max(tokens.values()) >= cfg.vocab_size:
        raise ValueError("vocabulary too small for the synthetic token contract")
    return tokens


def sha256_file(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def tokenizer_metadata(root, expected=None):
    """Checksums of the tokenizer files (and the special ids); raise if ``expected`` differs."""
    files = {name: sha256_file(Path(root) / name) for name in TOKENIZER_FILES if (Path(root) / name).exists()}
    if expected is not None:
        for name, digest in expected.get("files", {}).items():
            if files.get(name) != digest:
                raise ValueError(f"tokenizer checksum changed: {name}")
    return dict(files=files, counting=dict(exclude_special_token_ids=special_token_ids(root)))
