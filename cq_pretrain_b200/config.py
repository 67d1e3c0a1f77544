"""Run configuration: one flat dataclass assembled from model, data, loss and runtime groups.

Field names and defaults follow the reference's ``RunConfig`` so that checkpoint
``config`` dictionaries stay interchangeable (reference ``configs/config.py:13-158``).
Validation rules restate the reference's invariants (``configs/config.py:81-137,141-158``);
the B200 build adds ``gdn_backend='cuda'`` (the hand-written sm_100a kernels) and keeps the
reference's backend names loadable for old checkpoints.
"""

from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path

GDN_BACKENDS = ("cuda", "ascendc", "mindspeed")


@dataclass
class RuntimeConfig:
    gdn_backend: str = "cuda"
    ce_chunk: int = 256
    checkpoint_backbone: bool = False
    checkpoint_dit: bool = False
    checkpoint_backbone_layers: int = 0
    checkpoint_dit_layers: int = 0
    keep_attention_activations: int = 0
    fused: bool = True
    checkpoint_vision: bool = False


@dataclass
class ModelConfig(RuntimeConfig):
    method: str = "CQ_IT"
    content_visibility: str = "visual_block"
    image_condition_queries: int = 64
    visual_query_mode: str = "native"
    wan_assets: str = ""
    wan_vae_assets: str = ""
    wan_freq_dim: int = 256
    text_mask_token_id: int = 248063
    image_mask_token_id: int = 248056
    architecture: str = "qwen35_cq"
    text_assets: str = ""
    vocab_size: int = 248320
    width: int = 2048
    layers: int = 24
    heads: int = 8
    kv_heads: int = 2
    head_dim: int = 256
    ffn: int = 6144
    linear_value_heads: int = 0
    qwen_fused_projections: bool = True
    tie_word_embeddings: bool = True
    renderer: str = "wan"
    moss_assets: str = ""
    moss_fused_qkv: bool = False
    moss_cross_attention: bool = False
    linear_heads: int = 16
    linear_head_dim: int = 128
    linear_conv_kernel: int = 4
    full_attention_interval: int = 4
    partial_rotary_factor: float = 0.25
    mrope_section: tuple = (11, 11, 10)
    rope_theta: float = 10000000.0
    norm_eps: float = 1e-6
    image_size: int = 512
    patch_size: int = 16
    latent_channels: int = 16
    dit_width: int = 1536
    dit_heads: int = 12
    dit_layers: int = 30
    dit_ffn: int = 8960
    flow_draws: int = 1
    vision_encoder: str = "qwen35"
    vision_assets: str = ""
    freeze_vision: bool = True
    freeze_vision_merger: bool = True
    vision_tensor_parallel: bool = False

    # ---- derived geometry -------------------------------------------------------------
    @property
    def image_tokens(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    @property
    def value_heads(self) -> int:
        return self.linear_value_heads or self.linear_heads

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def dit_head_dim(self) -> int:
        return self.dit_width // self.dit_heads

    def is_attention_layer(self, index: int) -> bool:
        return (index + 1) % self.full_attention_interval == 0

    def validate_model(self, tp: int = 1) -> None:
        def need(ok, message):
            if not ok:
                raise ValueError(message)

        need(self.content_visibility in ("causal", "visual_block"), "content_visibility must be causal or visual_block")
        need(self.architecture == "qwen35_cq", "the backbone is the Qwen3.5 CQ hybrid")
        need(tp in (1, 2, 4, 8), "supported TP sizes: 1, 2, 4, 8")
        need(self.linear_heads % tp == 0 and self.value_heads % tp == 0, "GDN head counts must divide TP")
        need(self.value_heads % self.linear_heads == 0, "GDN grouped heads must be integral")
        need(self.full_attention_interval == 4, "Qwen3.5 CQ uses three GatedDeltaNet layers per gated-attention layer")
        need(min(self.linear_heads, self.linear_head_dim, self.linear_conv_kernel) >= 1, "invalid linear attention dims")
        need(self.rotary_dim % 2 == 0 and sum(self.mrope_section) == self.rotary_dim // 2,
             "MRoPE sections must cover the partial rotary dimensions")
        need(self.method in ("CQ_IT", "Bi_I+CQ_T"), "method must be CQ_IT or Bi_I+CQ_T")
        need(self.visual_query_mode in ("fixed", "native"), "visual_query_mode must be fixed or native")
        need(self.gdn_backend in GDN_BACKENDS, f"gdn_backend must be one of {GDN_BACKENDS}")
        need(self.renderer in ("wan", "legacy", "moss"), "renderer must be wan, legacy or moss")
        need(not ((self.renderer == "legacy" or self.vision_encoder == "rgb_patch") and tp > 1),
             "the legacy renderer and RGB patch embedding run replicated (TP = 1)")
        if self.renderer == "wan":
            need(self.flow_draws == 1 and self.latent_channels == 16, "Wan uses one flow draw and 16-channel latents")
        if self.renderer == "moss":
            need(self.flow_draws == 1, "the MOSS renderer trains one flow draw per target")
            need(self.dit_width % self.dit_heads == 0 and (self.dit_width // self.dit_heads) % 8 == 0,
                 "MOSS head width must be a multiple of 8 (four RoPE axes, rotate-half)")
            need(self.dit_heads % tp == 0 and self.dit_ffn % tp == 0, "MOSS heads and FFN width must divide TP")
        q = self.image_condition_queries
        need(q >= 1 and (self.renderer in ("wan", "moss") or math.isqrt(q) ** 2 == q),
             "image query count must be a positive square")
        need(self.vision_encoder in ("rgb_patch", "qwen35"), "vision_encoder must be rgb_patch or qwen35")
        need(not ((self.freeze_vision or self.freeze_vision_merger) and self.vision_encoder != "qwen35"),
             "vision freezing is defined for the Qwen vision encoder and merger")
        need(all(0 <= t < self.vocab_size for t in (self.text_mask_token_id, self.image_mask_token_id)),
             "mask embeddings must be valid vocabulary entries")
        need(self.image_size % self.patch_size == 0, "image_size must be divisible by patch_size")
        for name in ("heads", "kv_heads", "ffn", "dit_heads", "dit_ffn", "vocab_size"):
            need(getattr(self, name) % tp == 0, f"{name} must be divisible by TP={tp}")
        need(self.heads % self.kv_heads == 0 and self.head_dim % 4 == 0, "GQA ratio integral, head_dim % 4 == 0")
        need(self.dit_width % self.dit_heads == 0 and self.dit_head_dim % 4 == 0, "DiT head_dim must be divisible by four")
        need(min(self.layers, self.dit_layers, self.flow_draws, self.ce_chunk) >= 1, "layer, draw, chunk counts positive")
        need(0 <= self.checkpoint_backbone_layers <= self.layers, "invalid count of recomputed backbone layers")
        need(0 <= self.checkpoint_dit_layers <= self.dit_layers, "invalid count of recomputed DiT layers")
        need(0 <= self.keep_attention_activations <= self.layers // self.full_attention_interval,
             "invalid count of retained full-attention activations")


@dataclass
class DataConfig:
    visual_cache: str = ""
    generation_max_pixels: int = 1048576
    generation_token_budget: int = 8192
    preserve_documents: bool = False
    long_document_policy: str = "window"
    generation_microbatch_images: int = 0
    i2t_image_loss_probability: float = 1.0
    visual_uncond_probability: float = 0.1
    cfg_null_condition: str = "empty"
    vision_min_pixels: int = 65536
    vision_max_pixels: int = 1048576


@dataclass
class LossConfig:
    text_weight: float = 0.05
    image_weight: float = 1.0


@dataclass
class RunConfig(ModelConfig, DataConfig, LossConfig):
    def validate(self, tp: int = 1) -> "RunConfig":
        self.validate_model(tp)

        def need(ok, message):
            if not ok:
                raise ValueError(message)

        need(not self.generation_max_pixels or self.generation_max_pixels >= 256, "generation must fit one 16x16 cell")
        need(self.generation_token_budget >= 0 and self.generation_microbatch_images >= 0,
             "generation microbatch limits must be nonnegative")
        need(0 <= self.i2t_image_loss_probability <= 1, "I2T image loss probability must be in [0, 1]")
        need(0 <= self.visual_uncond_probability <= 1, "unconditional probability must be in [0, 1]")
        need(self.cfg_null_condition in ("empty", "empty_t2i", "i2t_prefix"), "unknown CFG null condition")
        need(not (self.renderer == "wan" and self.cfg_null_condition == "i2t_prefix"),
             "Wan understanding inputs have no generation queries")
        need(not (self.renderer == "wan" and self.visual_uncond_probability and self.cfg_null_condition != "empty"),
             "Wan unconditional training requires the empty query-read condition")
        need(self.long_document_policy in ("window", "error"), "long documents need a window or error policy")
        need(not (self.visual_cache and not (self.freeze_vision and self.freeze_vision_merger)),
             "a visual feature cache requires a frozen ViT and merger")
        need(1024 <= self.vision_min_pixels <= self.vision_max_pixels, "require 1024 <= vision_min <= vision_max pixels")
        return self

    # ---- (de)serialisation ------------------------------------------------------------
    @classmethod
    def from_dict(cls, values: dict) -> "RunConfig":
        known = {f.name for f in fields(cls)}
        unknown = set(values) - known
        if unknown:
            raise ValueError(f"unknown configuration fields: {sorted(unknown)}")
        values = dict(values)
        if "mrope_section" in values:
            values["mrope_section"] = tuple(values["mrope_section"])
        return cls(**values)

    @classmethod
    def load(cls, path) -> "RunConfig":
        """YAML with ``model/data/loss/runtime`` sections (flattened, duplicates rejected) or flat JSON."""
        path = Path(path)
        text = path.read_text()
        if path.suffix in (".yaml", ".yml"):
            import yaml

            value = yaml.safe_load(text) or {}
            if "model" not in value:
                return cls.from_dict({k: v for k, v in value.items() if k not in ("training", "environment")})
            flat: dict = {}
            for section in ("model", "data", "loss", "runtime"):
                for name, setting in (value.get(section) or {}).items():
                    if name in flat:
                        raise ValueError(f"duplicate configuration field: {name}")
                    flat[name] = setting
            return cls.from_dict(flat)
        return cls.from_dict(json.loads(text))

    def to_dict(self) -> dict:
        values = asdict(self)
        values["mrope_section"] = list(values["mrope_section"])
        return values


def load_sections(path) -> tuple[RunConfig, dict, dict]:
    """Return (config, training defaults, environment defaults) from a YAML run file."""
    import yaml

    raw = yaml.safe_load(Path(path).read_text()) or {}
    return RunConfig.load(path), dict(raw.get("training") or {}), dict(raw.get("environment") or {})


def tiny_config(**overrides) -> RunConfig:
    """The tiny joint model: a 4-layer hybrid (3 GDN + 1 attention) that runs on CPU in fp32."""
    values = dict(
        renderer="wan",
        vision_encoder="qwen35",
        freeze_vision=True,
        freeze_vision_merger=True,
        vocab_size=1024,
        width=256,
        layers=4,
        heads=4,
        kv_heads=2,
        head_dim=64,
        ffn=768,
        linear_heads=4,
        linear_head_dim=64,
        linear_conv_kernel=4,
        partial_rotary_factor=0.25,
        mrope_section=(3, 3, 2),
        image_size=256,
        patch_size=16,
        dit_width=128,
        dit_heads=4,
        dit_layers=2,
        dit_ffn=512,
        wan_freq_dim=64,
        ce_chunk=128,
        image_condition_queries=64,
        visual_query_mode="native",
        visual_uncond_probability=0.0,
        text_mask_token_id=4,
        image_mask_token_id=5,
        generation_token_budget=0,
    )
    values.update(overrides)
    return RunConfig(**values)


def qwen35_2b_wan(**overrides) -> RunConfig:
    """Qwen3.5-2B hybrid backbone + Wan2.1-T2V-1.3B (the reference production model)."""
    values = dict(ce_chunk=1024, generation_token_budget=65536, visual_uncond_probability=0.1,
                  preserve_documents=False)
    values.update(overrides)
    return RunConfig(**values)
