"""Document-aware packing into fixed-length CQ sequences, with consumed-only receipts.

Behaviour follows the reference packer for the Wan path (``data/packing.py:45-431``):

* every templated document opens with BOS and closes with EOS (EOS and BOI are supervised
  structural targets); text tokens are supervised unless the element says otherwise;
* images/videos are atomic: a visual that does not fit moves to the next pack;
* long documents continue in the next pack (``long_document_policy='window'``) with a fresh
  opener, or raise (``'error'``); ``preserve_documents`` starts a whole document in a fresh
  pack when it does not fit in the remainder;
* understanding documents (I2T/V2T) contribute no generation targets; a generation target
  may be drawn unconditional (non-CFG) with ``visual_uncond_probability`` by a sha256
  Bernoulli keyed on (seed, epoch, document, element), so prefetch depth and pack boundaries
  never change the draw;
* every pack carries a receipt; :class:`ConsumedLoader` only advances its resumable cursor
  when a receipt is acknowledged after a committed optimizer update.
"""

from __future__ import annotations

import copy
import hashlib
import math
from collections import deque
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from .batch import Batch, VisionInputs
from .generation import MossGenerationInputs, WanGenerationInputs
from .plan import build_plan, visual_query_count
from .sequence import image_sequence, video_sequence


def sample_objective(sample_id, probability, seed=0, epoch=0, salt="i2t-null-v1") -> bool:
    """Independent Bernoulli draw keyed by occurrence (stable across TP, prefetch and restart)."""
    if probability >= 1:
        return True
    if probability <= 0:
        return False
    digest = hashlib.sha256(f"{salt}:{seed}:{epoch}:{sample_id}".encode()).digest()
    return int.from_bytes(digest[:8], "big") < int(probability * (1 << 64))


DEFAULT_TOKENS = dict(bos=1, eos=2, boi=3, eoi=6, image=7, time=8)


def visual_layout(element, tokens):
    grid = tuple(element["grid"])
    if element.get("video") or grid[0] > 1:
        return video_sequence(grid, tokens)
    return image_sequence(grid, tokens)


def latent_dit_grid(element):
    """DiT token grid of a visual's generation latent ``[C, T, H, W]`` under the 1x2x2 patch."""
    c, t, h, w = element["latent_shape"]
    return t, h // 2, w // 2


class Packer:
    def __init__(self, documents, cfg, length, tokens=None, state=None, padding_multiple=0, pin=False,
                 row_multiple=1):
        if padding_multiple < 0:
            raise ValueError("padding multiple must be nonnegative")
        self.documents, self.cfg, self.length = documents, cfg, length
        self.tokens = dict(DEFAULT_TOKENS if tokens is None else tokens)
        self.tokens.setdefault("time", self.tokens["boi"])
        self.padding_multiple, self.pin, self.row_multiple = padding_multiple, pin, row_multiple
        self.element = self.offset = self.serial = 0
        self.contract = dict(preserve_documents=cfg.preserve_documents, long_document_policy=cfg.long_document_policy,
                             length=length, padding_multiple=padding_multiple, visual_query_mode=cfg.visual_query_mode,
                             visual_queries=cfg.image_condition_queries, visual_uncond_probability=cfg.visual_uncond_probability,
                             visibility="time_block_bidirectional_causal_v1")
        self.stats = dict(batches=0, long_document_windows=0, atomic_documents=0)
        if state:
            if state.get("packing") != self.contract:
                raise ValueError("document packing policy or limits differ on resume")
            self.element, self.offset, self.serial = state["element"], state["offset"], state["serial"]
            if "documents" in state and hasattr(documents, "load_state_dict"):
                documents.load_state_dict(state["documents"])

    def state_dict(self):
        docs = self.documents.state_dict() if hasattr(self.documents, "state_dict") else {}
        return dict(documents=docs, element=self.element, offset=self.offset, serial=self.serial,
                    packing=dict(self.contract))

    def _extent(self, doc):
        size = (2 if doc.get("templated", True) else 1)
        for e in doc["elements"]:
            size += len(e["input_ids"]) if e["type"] == "text" else len(visual_layout(e, self.tokens)["ids"])
        return size

    def next(self):
        s, cfg, t = self.length, self.cfg, self.tokens
        ids = np.full(s, t["eos"], np.int64)
        segment = np.full(s, -1, np.int64)
        sigma = np.arange(s, dtype=np.int64)
        rope = np.zeros((3, s), np.float32)
        image_queries = np.zeros(s, bool)
        text_indices, spans, grids, features, latent_grids, latents = [], [], [], [], [], []
        pixels = []
        gen_indices, gen_uncond = [], []
        records = []
        position = seg = body = 0
        while position < s:
            doc = self.documents.peek()
            if doc is None:
                break
            signature = getattr(self.documents, "signature", {})
            seed, epoch = signature.get("seed", 0), signature.get("epoch", 0)
            understanding = doc.get("direction") in ("I2T", "V2T")
            continued = bool(self.element or self.offset)
            if cfg.preserve_documents and not continued:
                needed = self._extent(doc)
                if needed > s:
                    if cfg.long_document_policy == "error":
                        raise ValueError(f"document {doc['id']} exceeds {s} tokens")
                    if position:
                        break
                elif position and s - position < needed:
                    break
                else:
                    self.stats["atomic_documents"] += 1
            elements = doc["elements"]
            while self.element < len(elements):  # skip exhausted/empty text elements
                e = elements[self.element]
                if e["type"] != "text" or self.offset < len(e["input_ids"]):
                    break
                self.element, self.offset = self.element + 1, 0
            first = elements[self.element] if self.element < len(elements) else None
            needed = (len(visual_layout(first, t)["ids"]) + 1) if (first and first["type"] == "image") else 2
            if position and s - position < needed:
                break
            start = position
            templated = doc.get("templated", True)
            cursor = 0
            if templated:
                ids[position], segment[position] = t["bos"], seg
                position += 1
                cursor = 1
            record = dict(id=doc["id"], element=self.element, offset=self.offset, body_tokens=0, images=0,
                          completed=False, window_continuation=continued)
            if continued:
                self.stats["long_document_windows"] += 1
            records.append(record)
            while self.element < len(elements) and position < s:
                e = elements[self.element]
                if e["type"] == "text":
                    take = min(len(e["input_ids"]) - self.offset, s - position)
                    if take:
                        ids[position:position + take] = np.asarray(e["input_ids"][self.offset:self.offset + take])
                        segment[position:position + take] = seg
                        rope[:, position:position + take] = np.arange(cursor, cursor + take)
                        if e.get("supervised", True):
                            text_indices.extend(range(position, position + take))
                        position += take
                        cursor += take
                        self.offset += take
                        body += take
                        record["body_tokens"] += take
                    if self.offset == len(e["input_ids"]):
                        self.element, self.offset = self.element + 1, 0
                    continue
                if e["type"] != "image":
                    raise ValueError(f"unsupported corpus element: {e['type']}")
                layout = visual_layout(e, t)
                size = len(layout["ids"])
                if position + size > s:
                    break
                stop = position + size
                ids[position:stop] = layout["ids"]
                segment[position:stop] = seg
                sigma[position:stop] = layout["sigma"] + position
                rope[:, position:stop] = layout["positions"] + cursor
                visual = position + layout["visual"]
                image_queries[visual] = True
                text_indices.extend((position + layout["text_indices"]).tolist())
                generate = (not understanding and e.get("generation_target", True) and "latent_shape" in e
                            and e.get("loss_allowed", True))
                unconditional = e.get("non_cfg", doc.get("non_cfg"))
                if unconditional is None:
                    unconditional = sample_objective(f"{doc['id']}:{self.element}", cfg.visual_uncond_probability,
                                                     seed, epoch, "visual-uncond-v1")
                if generate:
                    gen_indices.append(len(spans))
                    # MOSS latents are already 2x2-packed (16 pixels per token): grid = latent (h, w)
                    latent_grids.append(tuple(e["latent_shape"][-2:]) if cfg.renderer == "moss" else latent_dit_grid(e))
                    latents.append(e.get("latent"))
                gen_uncond.append(bool(generate and unconditional))
                spans.append(visual)
                grids.append(tuple(e["grid"]))
                features.append(e.get("features"))
                pixels.append(e.get("pixels"))
                cursor += int(layout["positions"].max()) + 1
                position = stop
                self.element += 1
                record["images"] += 1
            if self.element == len(elements) and position < s:
                ids[position], segment[position] = t["eos"], seg
                rope[:, position] = cursor
                text_indices.append(position)
                position += 1
                record["completed"] = True
                self.documents.advance()
                self.element = self.offset = 0
                seg += 1
            else:
                if position == start + (1 if templated else 0):
                    raise RuntimeError("packer made no progress; a visual element is larger than the pack")
                break
        if not records:
            return None
        if self.padding_multiple:
            used = min(s, math.ceil(position / self.padding_multiple) * self.padding_multiple)
            ids, segment, sigma, rope, image_queries = ids[:used], segment[:used], sigma[:used], rope[:, :used], image_queries[:used]
        n_vis = len(spans)
        width = max((len(x) for x in spans), default=0)
        indices = np.full((n_vis, width), -1, np.int64)
        for i, span in enumerate(spans):
            indices[i, :len(span)] = span
        vision = None
        if spans:
            feats = None
            if all(f is not None for f in features):
                feats = torch.cat([torch.as_tensor(f) for f in features])
            vision = VisionInputs(tuple(grids), torch.from_numpy(np.concatenate(spans)), feats)
            if pixels and all(px is not None for px in pixels):
                vision.pixel_values = torch.stack([torch.as_tensor(px).float() for px in pixels])
        batch = Batch(ids=torch.from_numpy(ids[None]), segments=torch.from_numpy(segment[None]),
                      sigma=torch.from_numpy(sigma[None]), positions=torch.from_numpy(rope),
                      text_indices=torch.tensor(sorted(text_indices), dtype=torch.long),
                      image_indices=torch.from_numpy(indices), image_queries=torch.from_numpy(image_queries[None]),
                      vision=vision, generation_image_indices=torch.tensor(gen_indices, dtype=torch.long),
                      generation_unconditional=torch.tensor(gen_uncond, dtype=torch.bool))
        if gen_indices and cfg.renderer == "legacy":
            # legacy flow renderer: one [tokens, C] latent grid per target (no 2x2 patching)
            if all(z is not None for z in latents):
                batch.latents = torch.stack([torch.as_tensor(z).float().reshape(z.shape[0], -1).T for z in latents])
        elif gen_indices and cfg.renderer == "moss":
            # MOSS: packed [latent tokens, conditions] streams; latents [C, (1,) h, w], 16 px per token
            counts = [visual_query_count(grids[i], cfg) for i in gen_indices]
            batch.generation = MossGenerationInputs.prepare(latent_grids, counts, cfg.dit_width // cfg.dit_heads,
                                                            cfg.generation_token_budget,
                                                            cfg.generation_microbatch_images)
            if all(z is not None for z in latents):
                batch.latents = torch.cat([torch.as_tensor(z).float().reshape(z.shape[0], -1).T for z in latents])
        elif gen_indices:
            counts = [visual_query_count(grids[i], cfg) for i in gen_indices]
            batch.generation = WanGenerationInputs.prepare(latent_grids, counts, cfg.dit_head_dim,
                                                           cfg.generation_token_budget, cfg.generation_microbatch_images)
            if all(z is not None for z in latents):
                from .generation import patch_latent
                batch.latents = torch.cat([patch_latent(torch.as_tensor(z).float()) for z in latents])
        batch.mainline = build_plan(batch, cfg, pad_multiple=self.row_multiple)
        if self.pin:
            batch = batch.pin_memory()
        self.serial += 1
        self.stats["batches"] += 1
        receipt = dict(serial=self.serial, next_state=self.state_dict(), documents=records, body_tokens=body,
                       occupied=position, images=n_vis, generation_images=len(gen_indices),
                       condition_query_tokens=int(batch.mainline.query_image.sum()),
                       unconditional_images=int(sum(gen_uncond)),
                       ids_sha256=hashlib.sha256(ids.tobytes()).hexdigest())
        return batch, receipt


class ConsumedLoader:
    """One bounded packing thread; the resumable state is the last *acknowledged* receipt.

    Checkpointing a prefetched loader therefore never skips unseen examples
    (reference ``data/packing.py:434-477``).
    """

    def __init__(self, packer, prefetch=2, state=None):
        if prefetch < 1:
            raise ValueError("prefetch must be positive")
        self.packer, self.limit = packer, prefetch
        self.pool = ThreadPoolExecutor(max_workers=1)
        self.pending, self.delivered = deque(), deque()
        self.consumed = copy.deepcopy(state or packer.state_dict())
        self.closed = False
        self._fill()

    def _fill(self):
        while not self.closed and len(self.pending) < self.limit:
            self.pending.append(self.pool.submit(self.packer.next))

    def next(self):
        if self.closed:
            return None
        result = self.pending.popleft().result()
        if result is None:
            self.closed = True
            return None
        self.delivered.append(result[1])
        self._fill()
        return result

    def acknowledge(self, receipt):
        expected = self.delivered[0]
        if receipt["serial"] != expected["serial"]:
            raise ValueError("consumption acknowledgements must arrive in order")
        self.delivered.popleft()
        self.consumed = copy.deepcopy(expected["next_state"])

    def state_dict(self):
        return copy.deepcopy(self.consumed)

    def close(self):
        self.closed = True
        self.pool.shutdown(wait=True, cancel_futures=True)
        if hasattr(self.packer.documents, "close"):
            self.packer.documents.close()
