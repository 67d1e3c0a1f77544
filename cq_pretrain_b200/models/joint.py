"""JointModel: CQ backbone executor, text cross-entropy and the Wan renderer.

``JointModel.forward(batch, return_hidden=False, compute_image_loss=True)`` returns the
*unweighted* ``text_loss`` and ``image_loss`` (``None`` without generation targets), plus
``image_conditions`` when the renderer loss is deferred to the chunked backward schedule
(reference ``models/modeling_umm.py:25-88``, ``models/cq_backbone.py:7-62``).

Backbone layout: ``hidden = [content rows (S); query rows (Q); padding]``. Content rows embed
the packed ids, with visual positions replaced by merger features; query rows embed the
image- or text-mask token. After the layers, the final RMSNorm output of the query rows is
scattered to ``output_positions`` (text queries at their own position, visual queries at
their condition slots after ``S``).
"""

from __future__ import annotations

import torch
from torch import nn

from ..data.batch import backbone_ids
from ..ops import cross_entropy as CE
from ..parallel import layers as PL
from ..parallel import state as ps
from .qwen35 import QwenBlock, RMSNorm
from .wan21 import Wan21Generator


class OutputHead(nn.Module):
    """Untied vocabulary-parallel LM head (used only by the text loss)."""

    def __init__(self, cfg):
        super().__init__()
        self.weight = PL.VocabEmbedding(cfg.vocab_size, cfg.width).weight


class JointModel(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        cfg.validate_model(ps.tp_size())
        self.cfg = cfg
        self.embedding = PL.VocabEmbedding(cfg.vocab_size, cfg.width)
        self.layers = nn.ModuleList([QwenBlock(cfg, i) for i in range(cfg.layers)])
        self.final_norm = RMSNorm(cfg.width, cfg.norm_eps)
        if cfg.renderer == "legacy":
            from .legacy import FlowRenderer
            self.renderer = FlowRenderer(cfg)
        elif cfg.renderer == "moss":
            from .moss import MOSSRenderer
            self.renderer = MOSSRenderer(cfg)
        else:
            self.renderer = Wan21Generator(cfg)
        self.lm_head = None if cfg.tie_word_embeddings else OutputHead(cfg)
        if cfg.vision_encoder == "qwen35":
            from .vision import VisionTower, vision_config
            self.patch_embed = VisionTower(vision_config(cfg), cfg.width, cfg.freeze_vision, cfg.freeze_vision_merger)
        elif cfg.vision_encoder == "rgb_patch":
            from .legacy import RGBPatchLinear
            self.patch_embed = RGBPatchLinear(cfg.width, cfg.patch_size)
        else:
            self.patch_embed = None

    # ---- backbone ---------------------------------------------------------------------------
    def embed(self, batch):
        """Row-sharded input hidden ``[rows/tp, width]`` for the packed sequence."""
        cfg = self.cfg
        all_ids = backbone_ids(batch, cfg.text_mask_token_id, cfg.image_mask_token_id)
        partial = self.embedding.partial(all_ids, batch.embed_plan)
        vision = batch.vision
        if vision is not None and vision.content_indices.numel():
            if vision.features is not None:
                feats = vision.features.to(partial.dtype)
            elif vision.layout is not None and self.patch_embed is not None:
                feats = self.patch_embed(vision.layout).to(partial.dtype)
            elif vision.pixel_values is not None and cfg.vision_encoder == "rgb_patch":
                pixels = vision.pixel_values.to(self.patch_embed.weight.dtype)
                feats = self.patch_embed(pixels).reshape(-1, cfg.width).to(partial.dtype)
            else:
                raise ValueError("visual content needs merger features (cached) or pixels for the vision tower")
            if ps.tp_size() > 1 and ps.tp_rank() != 0:
                feats = torch.zeros_like(feats)  # the row reduce-scatter sums partial lookups
            partial = partial.index_copy(0, vision.content_indices, feats)
        return PL.scatter_rows(partial)

    def backbone(self, batch, cache=None):
        cfg, plan = self.cfg, batch.mainline
        hidden = self.embed(batch)
        rope = (plan.rope_cos.to(hidden.dtype), plan.rope_sin.to(hidden.dtype))
        for index, layer in enumerate(self.layers):
            recompute = (cfg.checkpoint_backbone or index >= cfg.layers - cfg.checkpoint_backbone_layers)
            if cfg.is_attention_layer(index) and index // cfg.full_attention_interval < cfg.keep_attention_activations:
                recompute = False
            if cache is not None:
                hidden = layer(hidden, rope, plan, cache[index])
            elif recompute and self.training and torch.is_grad_enabled():
                hidden = torch.utils.checkpoint.checkpoint(layer, hidden, rope, plan, use_reentrant=False)
            else:
                hidden = layer(hidden, rope, plan)
        normed = PL.gather_rows(self.final_norm(hidden))
        s, q = plan.content_length, plan.queries
        query = normed[s:s + q]
        out = query.new_zeros(plan.output_size, cfg.width)
        return out.index_copy(0, plan.output_positions, query)

    # ---- objectives -------------------------------------------------------------------------
    def forward(self, batch, return_hidden=False, compute_image_loss=True):
        hidden = self.backbone(batch)
        image_loss = image_conditions = None
        if batch.generation_image_count:
            indices = batch.mainline.condition_indices
            if batch.generation_image_indices is not None:
                indices = indices.index_select(0, batch.generation_image_indices.to(indices.device))
            image_conditions = PL.replicated_use(hidden)[indices.clamp_min(0)]
            if compute_image_loss:
                image_loss = self.renderer(image_conditions, batch)
        targets = batch.ids.reshape(-1).index_select(0, batch.text_indices)
        if not targets.numel():
            text_loss = hidden.sum() * 0
        else:
            weight = self.embedding.weight if self.lm_head is None else self.lm_head.weight
            text_loss = CE.linear_cross_entropy(hidden.index_select(0, batch.text_indices), weight, targets,
                                                self.cfg.ce_chunk)
        result = dict(text_loss=text_loss, image_loss=image_loss)
        if return_hidden:
            result["hidden"] = hidden
        if not compute_image_loss:
            result["image_conditions"] = image_conditions
        return result
