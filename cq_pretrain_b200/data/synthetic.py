"""Synthetic document streams for the benchmark configurations (no corpus, no network).

Documents use the same element format as real corpora: text elements carry token ids, visual
elements carry a Qwen patch grid, synthetic merger features ``N(0,1)`` of the backbone width
and a Wan latent ``[16, T, H, W] ~ N(0,1)``. Every value derives from ``(seed, document index)``
so a stream is exactly resumable from its ``state_dict``.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .packing import Packer


class ListDocuments:
    """A finite, resumable list of documents (``peek``/``advance``/``state_dict``)."""

    def __init__(self, docs, signature=None):
        self.docs, self.index = list(docs), 0
        self.signature = signature or dict(snapshot="synthetic", seed=0, epoch=0, rank=0)

    def peek(self):
        return self.docs[self.index] if self.index < len(self.docs) else None

    def advance(self):
        self.index += 1

    def state_dict(self):
        return dict(index=self.index, signature=dict(self.signature))

    def load_state_dict(self, state):
        if state.get("signature", self.signature) != self.signature:
            raise ValueError("document stream signature differs on resume")
        self.index = state["index"]


def visual_element(cfg, rng, grid, latent_shape, generate=True, features=True, non_cfg=None):
    t, h, w = grid
    n = t * (h // 2) * (w // 2)
    element = dict(type="image", grid=tuple(grid), generation_target=generate)
    if features:
        element["features"] = torch.from_numpy(rng.standard_normal((n, cfg.width), dtype=np.float32))
    if latent_shape is not None:
        element["latent_shape"] = tuple(latent_shape)
        element["latent"] = torch.from_numpy(rng.standard_normal(latent_shape, dtype=np.float32))
    if non_cfg is not None:
        element["non_cfg"] = non_cfg
    if t > 1:
        element["video"] = True
    return element


def text_ids(rng, n, vocab, low=16):
    return rng.integers(low, vocab, size=n, dtype=np.int64)


def joint_pack_documents(cfg, length, images=2, seed=0, grid=(1, 32, 32), latent_shape=(16, 1, 64, 64),
                         doc_range=(64, 4096), caption=32, understanding=True):
    """Documents that fill one pack of ``length`` tokens: T2I captions (+ I2T) and log-uniform text docs.

    Production-model shape: each visual has ``grid`` Qwen patches (merged tokens = t*h*w/4) and a
    ``latent_shape`` Wan target; remaining space is text documents of log-uniform lengths in
    ``doc_range``; the last document is cut to fill the pack exactly.
    """
    rng = np.random.default_rng(seed)
    docs = []
    # understanding: True -> half of the visuals are I2T, "all" -> every visual is I2T
    half = images if understanding == "all" else (images // 2 if understanding and images > 1 else 0)
    for i in range(images):
        direction = "I2T" if i >= images - half else "T2I"
        cap = dict(type="text", input_ids=text_ids(rng, caption, cfg.vocab_size))
        vis = visual_element(cfg, rng, grid, latent_shape, generate=direction == "T2I")
        elements = [cap, vis] if direction == "T2I" else [vis, cap]
        docs.append(dict(id=f"visual-{seed}-{i}", elements=elements, direction=direction, format="caption"))
    used = sum(2 + sum(len(e["input_ids"]) if e["type"] == "text" else
                       (e["grid"][0] * (e["grid"][1] // 2) * (e["grid"][2] // 2) + 2) for e in d["elements"])
               for d in docs)
    lo, hi = math.log(doc_range[0]), math.log(doc_range[1])
    k = 0
    while used < length:
        n = int(round(math.exp(rng.uniform(lo, hi))))
        n = max(1, min(n, length - used - 2))
        docs.append(dict(id=f"text-{seed}-{k}", elements=[dict(type="text", input_ids=text_ids(rng, n, cfg.vocab_size))]))
        used += n + 2
        k += 1
    return docs


def video_pack_documents(cfg, length, seed=0, grid=(4, 30, 52), latent_shape=(16, 21, 60, 104), text=4096,
                         understanding=True):
    """The T2V + V2T workload: one T2V target (81 frames at 480x832 -> 32,760 DiT tokens; Qwen content 8
    frames -> 1,560 merged tokens and 1,560 queries), with ``understanding`` one V2T document of the
    same geometry (video, then its caption as the text target), plus ``text`` tokens of text
    documents."""
    rng = np.random.default_rng(seed)
    docs = [dict(id=f"video-{seed}", direction="T2V", format="caption",
                 elements=[dict(type="text", input_ids=text_ids(rng, 64, cfg.vocab_size)),
                           visual_element(cfg, rng, grid, latent_shape)])]
    if understanding:
        docs.append(dict(id=f"video-v2t-{seed}", direction="V2T", format="caption",
                         elements=[visual_element(cfg, rng, grid, latent_shape, generate=False),
                                   dict(type="text", input_ids=text_ids(rng, 64, cfg.vocab_size))]))
    lo, hi = math.log(64), math.log(4096)
    used, k = 0, 0
    while used < text:
        n = max(1, min(int(round(math.exp(rng.uniform(lo, hi)))), text - used))
        docs.append(dict(id=f"vtext-{seed}-{k}", elements=[dict(type="text", input_ids=text_ids(rng, n, cfg.vocab_size))]))
        used += n + 2
        k += 1
    return docs


def tiny_pack_documents(cfg, length=512, seed=0, images=2, grid=(1, 16, 16), latent_shape=(16, 1, 8, 8),
                        doc_range=(32, 256)):
    """The tiny-model workload: 512 ids, 2 images of 64 merged tokens, docs of 32-256 tokens."""
    rng = np.random.default_rng(seed)
    docs = []
    for i in range(images):
        docs.append(dict(id=f"tiny-vis-{seed}-{i}", direction="T2I", format="caption",
                         elements=[dict(type="text", input_ids=text_ids(rng, int(rng.integers(8, 24)), cfg.vocab_size)),
                                   visual_element(cfg, rng, grid, latent_shape)]))
    for k in range(64):
        n = int(rng.integers(doc_range[0], doc_range[1] + 1))
        docs.append(dict(id=f"tiny-text-{seed}-{k}", elements=[dict(type="text", input_ids=text_ids(rng, n, cfg.vocab_size))]))
    return docs


def synthetic_batch(cfg, length=512, seed=0, kind="tiny", pad_multiple=1, **kwargs):
    """One packed, planned batch (host memory) of a benchmark configuration shape."""
    maker = dict(tiny=tiny_pack_documents, joint=joint_pack_documents, video=video_pack_documents,
                 gdn=gdn_pack_documents)[kind]
    docs = maker(cfg, length, seed=seed, **kwargs)
    packer = Packer(ListDocuments(docs, dict(snapshot="synthetic", seed=seed, epoch=0, rank=0)), cfg, length,
                    row_multiple=pad_multiple)
    batch, receipt = packer.next()
    return batch, receipt


def gdn_pack_documents(cfg, length, images=2, seed=0, grid=(1, 32, 32), doc_length=1024, caption=32):
    """The GDN layer microbenchmark workload: T2I captions, then text documents of
    ``doc_length`` tokens (a packed document boundary every 1024 tokens) up to ``length``."""
    rng = np.random.default_rng(seed)
    docs = []
    for i in range(images):
        docs.append(dict(id=f"gdn-vis-{seed}-{i}", direction="T2I", format="caption",
                         elements=[dict(type="text", input_ids=text_ids(rng, caption, cfg.vocab_size)),
                                   visual_element(cfg, rng, grid, (16, 1, 8, 8))]))
    used = images * (caption + grid[0] * (grid[1] // 2) * (grid[2] // 2) + 4)
    k = 0
    while used < length:
        n = max(1, min(doc_length - 2, length - used - 2))
        docs.append(dict(id=f"gdn-text-{seed}-{k}", elements=[dict(type="text", input_ids=text_ids(rng, n, cfg.vocab_size))]))
        used += n + 2
        k += 1
    return docs


def decode_prompt(cfg, ids, length=None):
    """One unsupervised text document ``ids`` planned for CQ decoding: its last token is the
    placeholder of the first unknown token and the plan's only query reads it."""
    from .plan import build_plan
    doc = dict(id="prompt", elements=[dict(type="text", input_ids=np.asarray(ids), supervised=False)],
               templated=False)
    packer = Packer(ListDocuments([doc]), cfg, length or (len(ids) + 8))
    batch, _ = packer.next()
    s = len(ids)
    batch.ids, batch.segments = batch.ids[:, :s], batch.segments[:, :s]
    batch.sigma, batch.positions = batch.sigma[:, :s], batch.positions[:, :s]
    batch.image_queries = batch.image_queries[:, :s]
    batch.text_indices = torch.tensor([s - 1])
    batch.mainline = build_plan(batch, cfg)
    return batch
