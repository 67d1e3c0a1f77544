"""Inference: flow-matching image/video generation with CFG and CQ greedy captioning.

* ``generate``: CQ conditions for the visual queries of a T2I/T2V pack (the target pixels
  are invisible to their own queries, so their merger features are zeros), projected once
  and cached as per-block cross-attention K/V; Euler integration over shifted sigmas
  ``s = shift b / (1 + (shift-1) b)`` with optional classifier-free guidance against the
  empty (non-CFG) condition (reference ``evaluations/sampling.py:264-334``).
* ``caption``: prefill + CQ cached decoding with greedy argmax over the vocabulary-parallel
  LM head (TP all-gather of the local maxima, reference ``evaluations/sampling.py:204-260``).
* ``run_suite``: evaluates a list of cases sharded over DP ranks and writes JSON, the media
  (PNG / MP4 or animated WebP, ``eval/media.py``) and an HTML report; ``eval.media.reference_scores``
  gives the teacher-forced text NLL and flow MSE of a case's reference targets.
"""

from __future__ import annotations

import html
import json
from pathlib import Path

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..data.generation import time_features, unpatch_latent
from ..parallel import state as ps


def flow_sigmas(steps, shift=5.0):
    if steps < 1 or shift <= 0:
        raise ValueError("positive steps and shift required")
    base = torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float64)
    return shift * base / (1 + (shift - 1) * base)


@torch.no_grad()
def conditions(model, batch):
    """Visual-query hidden states ``[targets, max_q, width]`` of a planned generation pack."""
    if batch.vision is not None:
        n = batch.vision.content_indices.numel()
        batch.vision.features = torch.zeros(n, model.cfg.width, device=batch.ids.device,
                                            dtype=model.embedding.weight.dtype)
    hidden = model.backbone(batch)
    idx = batch.mainline.condition_indices
    if batch.generation_image_indices is not None:
        idx = idx.index_select(0, batch.generation_image_indices.to(idx.device))
    return hidden[idx.clamp_min(0)], batch.generation


@torch.no_grad()
def generate(model, batch, steps=30, shift=5.0, guidance=1.0, seed=1234, null_batch=None, decode=None):
    """Return generated latent patches ``[sum L, C*4]`` (and decoded visuals when ``decode`` is given)."""
    renderer = model.renderer
    cond, layout = conditions(model, batch)
    projected = renderer.project_conditions(cond, layout)
    kv = renderer.cache_condition_kv(projected)
    neg_projected = neg_kv = None
    if guidance != 1.0:
        if null_batch is None:
            raise ValueError("classifier-free guidance needs the empty-condition pack")
        ncond, nlayout = conditions(model, null_batch)
        neg_projected = renderer.project_conditions(ncond, nlayout)
        neg_kv = renderer.cache_condition_kv(neg_projected)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    device = cond.device
    latent = torch.randn(sum(layout.lengths), model.cfg.latent_channels * 4, generator=gen).to(device)
    sigmas = flow_sigmas(steps, shift)
    feats = time_features(sigmas[:-1].float(), model.cfg.wan_freq_dim).to(device)
    for i, (s0, s1) in enumerate(zip(sigmas[:-1], sigmas[1:])):
        layout_i = layout.__class__(**{**layout.__dict__, "time_features": feats[i:i + 1].expand(len(layout.lengths), -1)})
        v = renderer.predict(latent, cond, layout_i, projected, kv).float()
        if neg_projected is not None:
            u = renderer.predict(latent, cond, layout_i, neg_projected, neg_kv).float()
            v = u + guidance * (v - u)
        latent = latent + float(s1 - s0) * v
    if not torch.isfinite(latent).all():
        raise FloatingPointError("non-finite generated latent")
    result = dict(latent=latent, grids=layout.grids)
    if decode is not None:
        outs, start = [], 0
        for grid, n in zip(layout.grids, layout.lengths):
            outs.append(decode(unpatch_latent(latent[start:start + n], grid, model.cfg.latent_channels)))
            start += n
        result["visuals"] = outs
    return result


def greedy_token(model, hidden):
    """Argmax over the full vocabulary from this rank's shard (ties -> smallest id)."""
    weight = model.embedding.weight if model.lm_head is None else model.lm_head.weight
    logits = F.linear(hidden.reshape(1, -1).to(weight.dtype), weight).float().flatten()
    local = int(logits.argmax())
    pair = torch.tensor([float(logits[local].detach()), float(local + ps.tp_rank() * weight.shape[0])], device=hidden.device)
    if ps.tp_size() > 1:
        pairs = [torch.empty_like(pair) for _ in range(ps.tp_size())]
        dist.all_gather(pairs, pair, group=ps.state().tp_group)
    else:
        pairs = [pair]
    best = min((p.tolist() for p in pairs), key=lambda x: (-x[0], x[1]))
    return int(best[1])


@torch.no_grad()
def caption(model, prefill_batch, max_new_tokens=48, stops=()):
    from ..models.decoding import CQDecoder
    decoder = CQDecoder(model, prefill_batch, max_new_tokens)
    emitted, reason = [], "max_new_tokens"
    for step in range(max_new_tokens):
        token = greedy_token(model, decoder.hidden)
        if token in stops:
            reason = f"stop_token_{token}"
            break
        emitted.append(token)
        if step + 1 < max_new_tokens:
            decoder.advance(token)
    return dict(token_ids=emitted, stop_reason=reason)


def run_suite(model, cases, output, runner):
    """Evaluate ``cases`` sharded over DP ranks (case i on DP rank i mod dp; every TP rank of a DP
    group runs the same cases, as the TP collectives need); ``runner(model, case) -> dict``.

    A runner result may carry ``visuals`` (a list of ``[T, H, W, 3]`` pixel arrays) or ``latents``
    (``[C, T, H, W]``, written as previews when no decoder produced pixels): DP-rank leaders (TP
    rank 0) save them under ``output/media`` as PNG (one frame) or MP4 / animated WebP and the
    results list the file names. Rank 0 writes ``results.json`` and an HTML report that embeds the
    media."""
    from .media import latent_preview, save_visual
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    st = ps.state()
    mine = [c for i, c in enumerate(cases) if i % st.dp == st.dp_rank]
    rows = []
    for case in mine:
        try:
            result = dict(runner(model, case))
            visuals = result.pop("visuals", None)
            latents = result.pop("latents", None)
            media = []
            if st.tp_rank == 0:
                frames = visuals if visuals is not None else [latent_preview(x) for x in (latents or [])]
                for k, pixels in enumerate(frames):
                    written = save_visual(pixels, output / "media" / f"{case.get('id')}_{k}")
                    media.append(written.name)
            if media:
                result["media"] = media
                result["media_kind"] = "decoded" if visuals is not None else "latent preview"
            rows.append(dict(id=case.get("id"), task=case.get("task"), **result))
        except Exception as error:  # noqa: BLE001 - reported per case
            rows.append(dict(id=case.get("id"), task=case.get("task"), error=f"{type(error).__name__}: {error}"))
    gathered = [rows]
    if dist.is_initialized() and st.dp > 1:
        gathered = [None] * st.dp
        dist.all_gather_object(gathered, rows, group=st.dp_group)
    results = [r for part in gathered for r in part]
    if not dist.is_initialized() or dist.get_rank() == 0:
        (output / "results.json").write_text(json.dumps(results, indent=2, default=str))
        def media_html(r):
            tags = []
            for name in r.get("media", []):
                src = html.escape(f"media/{name}")
                tags.append(f"<video src='{src}' controls loop></video>" if name.endswith(".mp4")
                            else f"<img src='{src}' style='max-width:320px'>")
            return "".join(tags)

        body = "".join(f"<section><h3>{html.escape(str(r.get('id')))} ({html.escape(str(r.get('task')))})</h3>"
                       f"{media_html(r)}"
                       f"<pre>{html.escape(json.dumps({k: v for k, v in r.items() if k not in ('id', 'task')}, default=str))}</pre></section>"
                       for r in results)
        (output / "report.html").write_text(f"<!doctype html><meta charset='utf-8'><title>CQ validation</title>{body}")
    return results
