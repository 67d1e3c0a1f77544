"""MOSS-Image-Base renderer (legacy) conditioned on CQ visual-query hidden states.

Architecture of the published MOSS-Image-Base DiT as the reference trains it
(``models/moss.py:24-314``):

* ``text_embedder``: Linear(backbone width -> dit width) and two refinement blocks (RMSNorm ->
  fused QKV with per-head Q/K RMSNorm and RoPE -> attention within each target's conditions ->
  RMSNorm -> SITU FFN);
* a shared time embedding (Linear 256 -> d, SiLU, Linear d -> d) and ONE shared 6-way block
  modulation (shift / scale / gate for attention and FFN) plus a 2-way head modulation;
* blocks over packed streams ``[noisy latent tokens, conditions]`` of each target: modulated
  RMSNorm -> Q/K/V (separate or fused) -> per-head Q/K RMSNorm -> four-axis RoPE -> attention
  within the stream -> gated residual -> (optional) cross-attention of latent tokens to their
  own conditions (ungated residual, no RoPE; the stream then carries latent tokens only) ->
  modulated RMSNorm -> SITU FFN -> gated residual;
* final RMSNorm, head modulation and a bias-free linear to the latent channels;
* flow matching with one draw per target: ``x_t = (1 - s) x0 + s eps``, velocity target
  ``eps - x0``, loss = sum over latent tokens of ``weight * mean_channels (v - target)^2``.

SITU, the affine modulation and the gated residual are the fused kernels of
``ops/activation.py`` (``csrc/moss.cu``). TP is Megatron style on replicated activations (column
shards for Q/K/V and the FFN up/gate projections, row shards for the output projections, each
rank attending with its own heads); the replicated norms and modulation layers hold full
gradients on every rank (``tp_duplicate``) except the per-head Q/K norms, which see only the local
heads and are summed over TP like sequence-parallel replicated parameters.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
from torch import nn

from ..ops import activation as A
from ..ops import attention as ATT
from ..ops import reference as R
from ..parallel import layers as P
from ..parallel import state as ps

MOSS_MODEL = ("OpenMOSS-Team/MOSS-Image-Base", "1ceede80badddd6a7812069619edaa5633587192")


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


def _per_head(norm, x, heads):
    return norm(x.unflatten(-1, (heads, -1))).flatten(-2)


def _attend(q, k, v, heads, q_ends, k_ends, rope=None):
    hd = q.shape[-1] // heads
    q, k, v = (t.reshape(t.shape[0], heads, hd) for t in (q, k, v))
    if rope is not None:
        q = R.rotary_half(q, rope[0], rope[1], hd)
        k = R.rotary_half(k, rope[0], rope[1], hd)
    y = ATT.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), q_ends, k_ends)
    return y.reshape(y.shape[0], heads * hd)


def _local_heads(heads):
    if heads % ps.tp_size():
        raise ValueError(f"MOSS heads {heads} not divisible by TP={ps.tp_size()}")
    return heads // ps.tp_size()


class TextBlock(nn.Module):
    def __init__(self, dim, ffn_dim, heads):
        super().__init__()
        self.heads = _local_heads(heads)
        self.norm1, self.norm2 = RMSNorm(dim), RMSNorm(dim)
        self.q_norm, self.k_norm = RMSNorm(dim // heads), RMSNorm(dim // heads)
        self.qkv = P.column_linear(dim, 3 * dim, stride=3)
        self.proj = P.row_linear(dim, dim)
        self.ffn_gate = P.column_linear(dim, ffn_dim)
        self.ffn_up = P.column_linear(dim, ffn_dim)
        self.ffn_down = P.row_linear(ffn_dim, dim)

    def forward(self, x, rope, ends):
        q, k, v = P.apply_column(self.qkv, self.norm1(x)).chunk(3, -1)
        q, k = _per_head(self.q_norm, q, self.heads), _per_head(self.k_norm, k, self.heads)
        x = x + P.apply_row(self.proj, _attend(q, k, v, self.heads, ends, ends, rope))
        y = self.norm2(x)
        hidden = A.situ(P.apply_column(self.ffn_up, y), P.apply_column(self.ffn_gate, y))
        return x + P.apply_row(self.ffn_down, hidden)


class TextProjection(nn.Module):
    def __init__(self, text_dim, dim, ffn_dim, heads):
        super().__init__()
        self.proj = nn.Linear(text_dim, dim)
        self.blocks = nn.ModuleList([TextBlock(dim, ffn_dim, heads) for _ in range(2)])

    def forward(self, x, rope, ends):
        x = self.proj(x.to(self.proj.weight.dtype))
        for block in self.blocks:
            x = block(x, rope, ends)
        return x


class CrossAttention(nn.Module):
    """Latent tokens (queries) read their own target's conditions; no RoPE; ungated residual."""

    def __init__(self, dim, heads):
        super().__init__()
        self.heads = _local_heads(heads)
        self.norm_q, self.norm_kv = RMSNorm(dim), RMSNorm(dim)
        self.q_norm, self.k_norm = RMSNorm(dim // heads), RMSNorm(dim // heads)
        self.to_q = P.column_linear(dim, dim, bias=False)
        self.to_kv = P.column_linear(dim, 2 * dim, bias=False, stride=2)
        self.to_out = P.row_linear(dim, dim, bias=False)

    def forward(self, x, memory, layout):
        q = _per_head(self.q_norm, P.apply_column(self.to_q, self.norm_q(x)), self.heads)
        k, v = P.apply_column(self.to_kv, self.norm_kv(memory)).chunk(2, -1)
        k = _per_head(self.k_norm, k, self.heads)
        return x + P.apply_row(self.to_out, _attend(q, k, v, self.heads, layout.video_ends, layout.text_ends))


class Block(nn.Module):
    def __init__(self, dim, ffn_dim, heads, fused_qkv=False, cross=False):
        super().__init__()
        self.heads = _local_heads(heads)
        self.fused_qkv = fused_qkv
        self.cross_attn = CrossAttention(dim, heads) if cross else None
        self.norm1, self.norm2 = RMSNorm(dim), RMSNorm(dim)
        self.q_norm, self.k_norm = RMSNorm(dim // heads), RMSNorm(dim // heads)
        proj = {"qkv": P.column_linear(dim, 3 * dim, bias=False, stride=3)} if fused_qkv else \
            {name: P.column_linear(dim, dim, bias=False) for name in ("q", "k", "v")}
        proj["o"] = P.row_linear(dim, dim, bias=False)
        proj["ffn_up_gate"] = P.column_linear(dim, 2 * ffn_dim, bias=False, stride=2)
        proj["ffn_down"] = P.row_linear(ffn_dim, dim, bias=False)
        self.proj = nn.ModuleDict(proj)

    def forward(self, x, rope, modulation, ends, memory=None, layout=None):
        shift_a, scale_a, gate_a, shift_f, scale_f, gate_f = modulation
        y = A.affine(self.norm1(x), scale_a, shift_a)
        if self.fused_qkv:
            q, k, v = P.apply_column(self.proj["qkv"], y).chunk(3, -1)
        else:
            q, k, v = (P.apply_column(self.proj[name], y) for name in ("q", "k", "v"))
        q, k = _per_head(self.q_norm, q, self.heads), _per_head(self.k_norm, k, self.heads)
        x = A.gated_add(x, P.apply_row(self.proj["o"], _attend(q, k, v, self.heads, ends, ends, rope)), gate_a)
        if self.cross_attn is not None:
            x = self.cross_attn(x, memory, layout)
        y = A.affine(self.norm2(x), scale_f, shift_f)
        hidden, gate = P.apply_column(self.proj["ffn_up_gate"], y).chunk(2, -1)
        return A.gated_add(x, P.apply_row(self.proj["ffn_down"], A.situ(hidden, gate)), gate_f)


class Rope(nn.Module):
    def __init__(self, head_dim):
        super().__init__()
        n = head_dim // 8
        self.register_buffer("bands", 1 / (10000 ** (torch.arange(n, dtype=torch.float32) / n)))


class MOSSRenderer(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        dim, ffn, heads = cfg.dit_width, cfg.dit_ffn, cfg.dit_heads
        self.video_embedder = nn.Linear(cfg.latent_channels, dim)
        self.text_embedder = TextProjection(cfg.width, dim, ffn, heads)
        self.rope = Rope(dim // heads)
        self.time_embedding = nn.Sequential(nn.Linear(256, dim), nn.SiLU(), nn.Linear(dim, dim))
        self.shared_block_modulation = nn.Linear(dim, 6 * dim)
        self.cross_conditioning = bool(cfg.moss_cross_attention)
        self.layers = nn.ModuleList([Block(dim, ffn, heads, cfg.moss_fused_qkv, self.cross_conditioning)
                                     for _ in range(cfg.dit_layers)])
        self.final_norm_video = RMSNorm(dim)
        self.final_linear_video = nn.Linear(dim, cfg.latent_channels, bias=False)
        self.video_head_modulation = nn.Linear(dim, 2 * dim)
        self.initialize_cross_attention()
        P.mark_duplicates(self)
        # per-head Q/K norms see only this rank's heads: partial gradients, summed over TP
        for name, p in self.named_parameters():
            if name.endswith("q_norm.weight") or name.endswith("k_norm.weight"):
                p.tp_duplicate = False

    # ---- conditioning -----------------------------------------------------------------------
    def project_conditions(self, conditions, layout, rope=None):
        dtype = self.video_embedder.weight.dtype
        rope = (layout.cos.to(dtype), layout.sin.to(dtype)) if rope is None else rope
        text_rope = tuple(t.index_select(0, layout.text_indices) for t in rope)
        flat = conditions.reshape(-1, conditions.shape[-1])
        if flat.shape[0] != layout.text_indices.numel():
            # conditions [n, max_q, width] with fewer queries for some targets
            width = conditions.shape[1]
            rows = torch.cat([torch.arange(q, device=flat.device) + i * width
                              for i, q in enumerate(layout.query_counts)])
            flat = flat.index_select(0, rows)
        return self.text_embedder(flat, text_rope, layout.text_ends)

    def predict(self, xt, conditions, time_features, layout, projected=None):
        cfg, dtype = self.cfg, self.video_embedder.weight.dtype
        time = self.time_embedding(time_features.to(dtype)).float()
        mod = self.shared_block_modulation(time.to(dtype)).view(-1, 6, cfg.dit_width)
        modulation = tuple(m.contiguous() for m in mod.index_select(0, layout.sample_indices).unbind(1))
        head = self.video_head_modulation(time.to(dtype)).view(-1, 2, cfg.dit_width)
        rope = (layout.cos.to(dtype), layout.sin.to(dtype))
        text = self.project_conditions(conditions, layout, rope) if projected is None else projected
        video = self.video_embedder(xt.to(dtype))
        if self.cross_conditioning:
            # latent tokens attend among themselves; conditions arrive through cross-attention
            x, ends = video, layout.video_ends
            modulation = tuple(m.index_select(0, layout.video_indices).contiguous() for m in modulation)
            rope = tuple(t.index_select(0, layout.video_indices) for t in rope)
        else:
            x = video.new_zeros(layout.ends[-1], cfg.dit_width)
            x = x.index_copy(0, layout.video_indices, video).index_copy(0, layout.text_indices, text)
            ends = layout.ends
        for index, layer in enumerate(self.layers):
            recompute = cfg.checkpoint_dit or index >= cfg.dit_layers - cfg.checkpoint_dit_layers
            if self.training and torch.is_grad_enabled() and recompute:
                x = torch.utils.checkpoint.checkpoint(layer, x, rope, modulation, ends, text, layout,
                                                      use_reentrant=False)
            else:
                x = layer(x, rope, modulation, ends, text, layout)
        if not self.cross_conditioning:
            x = x.index_select(0, layout.video_indices)
        x = self.final_norm_video(x)
        head = head.index_select(0, layout.video_sample_indices)
        x = A.affine(x, head[:, 1].contiguous(), head[:, 0].contiguous())
        return self.final_linear_video(x)

    def forward(self, conditions, batch):
        if self.cfg.flow_draws != 1:
            raise ValueError("the MOSS renderer trains exactly one flow draw per target")
        layout = batch.generation
        sigma = batch.times.index_select(0, layout.video_sample_indices)[:, None].float()
        target, noise = batch.latents.float(), batch.noise.float()
        xt = (1 - sigma) * target + sigma * noise
        prediction = self.predict(xt, conditions, layout.time_features, layout)
        mse = (prediction.float() - (noise - target)).square().mean(-1)
        return (mse * layout.loss_weights.to(mse.device)).sum()

    # ---- weights ----------------------------------------------------------------------------
    def official_tensors(self):
        """Writable views under the published MOSS checkpoint names (cross-attention, which the
        published model lacks, is excluded; a fused QKV weight maps to its q / k / v parts)."""
        target = {}
        for name, tensor in self.named_parameters():
            if ".cross_attn." in name:
                continue
            if name.endswith(".proj.qkv.weight") or name.endswith(".proj.qkv.bias"):
                for label, part in zip(("q", "k", "v"), tensor.chunk(3, dim=0)):
                    if getattr(tensor, "tensor_model_parallel", False):
                        P.mark_sharded(part)
                    target[name.replace(".qkv.", f".{label}.")] = part
            else:
                target[name] = tensor
        target["rope.bands"] = self.rope.bands
        return target

    def initialize_cross_attention(self):
        """Normal(0.02) for the added projections, output std scaled by 1/sqrt(2 depth); every rank
        draws the same full matrix and keeps its TP slice. Returns the number initialised."""
        if not self.cross_conditioning:
            return 0
        count = 0
        with torch.no_grad():
            for layer in self.layers:
                for name in ("to_q", "to_kv", "to_out"):
                    weight = getattr(layer.cross_attn, name).weight
                    std = 0.02 / (2 * self.cfg.dit_layers) ** 0.5 if name == "to_out" else 0.02
                    shape = list(weight.shape)
                    if getattr(weight, "tensor_model_parallel", False):
                        shape[weight.partition_dim] *= ps.tp_size()
                    value = torch.empty(shape, dtype=torch.float32).normal_(std=std)
                    weight.copy_(P.checkpoint_shard(value, weight))
                    count += 1
        return count

    def load_pretrained(self, path):
        """Load the pinned published checkpoint (``manifest.json`` + sharded safetensors)."""
        from safetensors import safe_open
        root = Path(path)
        manifest = json.loads((root / "manifest.json").read_text())
        if (manifest.get("model_id"), manifest.get("revision")) != MOSS_MODEL:
            raise ValueError("unexpected MOSS checkpoint (model id / revision pin)")
        index = json.loads((root / "transformer/diffusion_pytorch_model.safetensors.index.json").read_text())["weight_map"]
        target = self.official_tensors()
        if set(target) != set(index):
            raise ValueError(f"MOSS key mismatch: missing={sorted(set(index) - set(target))[:8]}, "
                             f"extra={sorted(set(target) - set(index))[:8]}")
        with torch.no_grad():
            for shard in sorted(set(index.values())):
                with safe_open(str(root / "transformer" / shard), framework="pt", device="cpu") as source:
                    for name, tensor in target.items():
                        if index[name] != shard:
                            continue
                        value = P.checkpoint_shard(source.get_tensor(name), tensor)
                        if value.shape != tensor.shape:
                            raise ValueError(f"MOSS shape mismatch: {name}: {tuple(value.shape)} vs {tuple(tensor.shape)}")
                        tensor.copy_(value)
        return dict(model_id=manifest["model_id"], revision=manifest["revision"], loaded_tensors=len(target))
