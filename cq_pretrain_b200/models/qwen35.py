"""Qwen3.5 hybrid decoder blocks with CQ read-only query streams.

Three Gated-DeltaNet blocks per gated full-attention block (reference
``models/backbone_qwen35.py:13-344``). Parameter names match the official Qwen3.5 layout
(fused ``in_proj_all`` / ``gate_up_proj`` / ``kv_proj`` when ``qwen_fused_projections``), so
``unfused_parameters`` can expose official tensor views.

Every block takes and returns row-sharded hidden states ``[rows/tp, width]`` (sequence
parallel). Column projections gather rows; the GDN recurrence and attention run on all rows
for this rank's heads; row projections scatter back.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import activation as A
from ..ops import attention as ATT
from ..ops import gather as GA
from ..ops import gdn as GDN
from ..ops import norms as N
from ..ops import reference as R
from ..ops import rope as ROPE
from ..parallel import layers as PL
from ..parallel import state as ps


class RMSNorm(nn.Module):
    """RMSNorm storing the offset from one (Qwen3.5 checkpoints, including Q/K norms)."""

    def __init__(self, width, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(width))
        self.eps = eps

    def forward(self, x):
        if x.dtype == torch.float64:
            return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + self.eps) * (1 + self.weight)
        return N.rms_norm(x, self.weight, self.eps)

    def residual(self, x):
        """``(x, norm(x))`` for an ``x`` that also continues along the residual stream: on CUDA the
        backward adds the residual gradient inside the norm's backward kernel."""
        if x.dtype == torch.float64:
            return x, self(x)
        return N.rms_norm_residual(x, self.weight, self.eps)

    def residual_add(self, x, branch):
        """``(x + branch, norm(x + branch))``: the residual add fused into the norm on CUDA."""
        if x.dtype == torch.float64:
            s = x + branch
            return s, self(s)
        return N.add_rms_norm_residual(x, branch, self.weight, self.eps)


class MLP(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.fused = cfg.qwen_fused_projections
        if self.fused:
            self.gate_up_proj = PL.ColumnLinear(cfg.width, 2 * cfg.ffn, stride=2)
        else:
            self.gate_proj = PL.ColumnLinear(cfg.width, cfg.ffn)
            self.up_proj = PL.ColumnLinear(cfg.width, cfg.ffn)
        self.down_proj = PL.RowLinear(cfg.ffn, cfg.width)

    def forward(self, x):
        if self.fused:
            return self.down_proj(A.swiglu(self.gate_up_proj(x)))
        if ps.tp_size() > 1:
            xg = PL.gather_rows(x)
            return self.down_proj(F.silu(self.gate_proj(xg, gathered=True)) * self.up_proj(xg, gathered=True))
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class CausalConv(nn.Module):
    def __init__(self, channels, kernel):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(channels, 1, kernel))
        nn.init.uniform_(self.weight, -0.5, 0.5)

    def forward(self, x, bounds):
        return GDN.causal_conv_silu(x, self.weight[:, 0], bounds)


class GatedNorm(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x, z):
        if x.dtype == torch.float64:
            normed = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + self.eps)
            return normed * self.weight * F.silu(z)
        return N.gated_rms_norm(x, z, self.weight, self.eps)


class GatedDelta(nn.Module):
    """Gated DeltaNet mixer over the CQ event stream of a packed sequence."""

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        tp = ps.tp_size()
        key = cfg.linear_heads * cfg.linear_head_dim
        h = cfg.value_heads
        value = h * cfg.linear_head_dim
        if cfg.qwen_fused_projections:
            self.in_proj_all = PL.ColumnLinear(cfg.width, 2 * key + 2 * value + 2 * h,
                                               splits=(key, key, value, value, h, h))
        else:
            self.in_proj_qkv = PL.ColumnLinear(cfg.width, 2 * key + value, splits=(key, key, value))
            self.in_proj_z = PL.ColumnLinear(cfg.width, value)
            self.in_proj_a = PL.ColumnLinear(cfg.width, h)
            self.in_proj_b = PL.ColumnLinear(cfg.width, h)
        self.conv1d = CausalConv((2 * key + value) // tp, cfg.linear_conv_kernel)
        PL.mark_sharded(self.conv1d.weight, splits=(key, key, value))
        self.A_log = PL.mark_sharded(nn.Parameter(torch.rand(h // tp).mul(15.99).add(0.01).log()))
        self.dt_bias = PL.mark_sharded(nn.Parameter(torch.ones(h // tp)))
        self.norm = GatedNorm(cfg.linear_head_dim, cfg.norm_eps)
        self.out_proj = PL.RowLinear(value, cfg.width)

    def project(self, x):
        cfg, tp = self.cfg, ps.tp_size()
        size = cfg.linear_heads * cfg.linear_head_dim // tp
        h = cfg.value_heads // tp
        d = cfg.linear_head_dim
        if cfg.qwen_fused_projections:
            return self.in_proj_all(x).split((2 * size + h * d, h * d, h, h), -1)
        xg = PL.gather_rows(x) if tp > 1 else x
        return (self.in_proj_qkv(xg, gathered=True), self.in_proj_z(xg, gathered=True),
                self.in_proj_a(xg, gathered=True), self.in_proj_b(xg, gathered=True))

    def forward(self, x, plan, cache=None):
        cfg, tp = self.cfg, ps.tp_size()
        hk = cfg.linear_heads // tp
        h = cfg.value_heads // tp
        d = cfg.linear_head_dim
        size = hk * d
        raw, z, a, b = self.project(x)                      # full rows, local heads
        dp = plan.delta
        # updates: content rows in write order. The query conv reads each query's own projection
        # and the previous k-1 real content inputs of its document; queries never enter any other
        # token's history.
        updates, conv, query = GDN.conv_and_query(raw, self.conv1d.weight[:, 0], dp, size)
        q, k, v = conv.split((size, size, h * d), -1)
        q, k, query = q.reshape(-1, hk, d), k.reshape(-1, hk, d), query.reshape(-1, hk, d)
        v = v.reshape(-1, h, d)
        if h != hk:
            q, k, query = (t.repeat_interleave(h // hk, dim=1) for t in (q, k, query))
        # event order: content and query conv outputs feed reads; index nc (write of a read-only
        # event) gathers zeros
        q = GA.rows(q, dp.event_q, dp.event_q_inv, second=query)
        k = GA.rows(k, dp.event_write, dp.event_write_inv)
        v = GA.rows(v, dp.event_write, dp.event_write_inv)
        ctrl = torch.float64 if x.dtype == torch.float64 else torch.float32
        a = GA.rows(a, dp.content_order, dp.content_order_inv).to(ctrl)
        g = -self.A_log.to(ctrl).exp() * F.softplus(a + self.dt_bias.to(ctrl))
        beta = GA.rows(b, dp.content_order, dp.content_order_inv).to(ctrl).sigmoid()
        g = GA.rows(g.contiguous(), dp.event_write, dp.event_write_inv)
        beta = GA.rows(beta.contiguous(), dp.event_write, dp.event_write_inv)
        if cache is not None:
            if torch.is_grad_enabled():
                raise ValueError("CQ state caching is inference-only")
            y, state = GDN.prefill(q, k, v, g, beta, dp.event_bounds)
            cache["state"] = state  # [docs, H, Dk, Dv]
            count = cfg.linear_conv_kernel - 1
            hist = raw.new_zeros(count, raw.shape[-1])
            tail = updates[max(0, len(updates) - 1 - count):-1]
            if len(tail):
                hist[-len(tail):] = tail
            cache["conv"] = hist
            y = y.to(v.dtype)
        else:
            y = GDN.gated_delta(q, k, v, g, beta, dp.event_bounds)
        selected = GA.rows(y.contiguous(), dp.hidden_event, dp.hidden_event_inv).to(x.dtype)   # sentinel -> zeros
        out = self.norm(selected, z.reshape(-1, h, d)).flatten(-2)
        return self.out_proj(out)


class GatedAttention(nn.Module):
    """Gated full attention (q + sigmoid output gate, per-head q/k RMSNorm, partial MRoPE, GQA)."""

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        self.q_proj = PL.ColumnLinear(cfg.width, 2 * cfg.heads * cfg.head_dim)
        if cfg.qwen_fused_projections:
            self.kv_proj = PL.ColumnLinear(cfg.width, 2 * cfg.kv_heads * cfg.head_dim, stride=2)
        else:
            self.k_proj = PL.ColumnLinear(cfg.width, cfg.kv_heads * cfg.head_dim)
            self.v_proj = PL.ColumnLinear(cfg.width, cfg.kv_heads * cfg.head_dim)
        self.o_proj = PL.RowLinear(cfg.heads * cfg.head_dim, cfg.width)
        self.q_norm = RMSNorm(cfg.head_dim, cfg.norm_eps)
        self.k_norm = RMSNorm(cfg.head_dim, cfg.norm_eps)

    def forward(self, x, rope, plan, cache=None):
        cfg, tp = self.cfg, ps.tp_size()
        s = plan.content_length
        hq, hkv, hd = cfg.heads // tp, cfg.kv_heads // tp, cfg.head_dim
        if cfg.qwen_fused_projections:
            # q/gate over all rows and k/v over the content rows share one in-kernel all-gather
            qg, kv = PL.column_pair(x, self.q_proj, self.kv_proj, rows2=s)
            q, gate = qg.reshape(-1, hq, 2 * hd).chunk(2, -1)
            # kv_proj = [k_proj; v_proj] (all key heads, then all value heads)
            k, v = (t.reshape(s, hkv, hd) for t in kv.chunk(2, -1))
        else:
            xg = PL.gather_rows(x) if tp > 1 else x
            q, gate = self.q_proj(xg, gathered=True).reshape(-1, hq, 2 * hd).chunk(2, -1)
            k = self.k_proj(xg[:s], gathered=True).reshape(s, hkv, hd)
            v = self.v_proj(xg[:s], gathered=True).reshape(s, hkv, hd)
        q = self.q_norm(q)
        k = self.k_norm(k)
        cos, sin = rope
        q = ROPE.rotary_half(q, cos, sin, cfg.rotary_dim)
        k = ROPE.rotary_half(k, cos[:s], sin[:s], cfg.rotary_dim)
        if cache is not None:
            if torch.is_grad_enabled():
                raise ValueError("CQ state caching is inference-only")
            cache["k"], cache["v"] = k.detach().clone(), v.contiguous().clone()
        y = ATT.cq_attention(q, k, v.contiguous(), plan.attn_kstart, plan.attn_kend)
        return self.o_proj((y * gate.sigmoid().to(y.dtype)).flatten(-2))


class QwenBlock(nn.Module):
    def __init__(self, cfg, index):
        super().__init__()
        self.cfg = cfg
        self.input_layernorm = RMSNorm(cfg.width, cfg.norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.width, cfg.norm_eps)
        if cfg.is_attention_layer(index):
            self.self_attn = GatedAttention(cfg)
        else:
            self.linear_attn = GatedDelta(cfg)
        self.mlp = MLP(cfg)

    def forward(self, hidden, rope, plan, cache=None):
        hidden, normed = self.input_layernorm.residual(hidden)
        if hasattr(self, "linear_attn"):
            mixed = self.linear_attn(normed, plan, cache)
        else:
            mixed = self.self_attn(normed, rope, plan, cache)
        hidden, normed = self.post_attention_layernorm.residual_add(hidden, mixed)
        return hidden + self.mlp(normed)


def unfused_parameters(name, tensor, cfg):
    """Official-name views of fused projections (for checkpoint loading and gradient checks)."""
    tp = ps.tp_size()
    if name.endswith(".mlp.gate_up_proj.weight"):
        return dict(zip((name.replace("gate_up_proj", "gate_proj"), name.replace("gate_up_proj", "up_proj")),
                        tensor.chunk(2, 0)))
    if name.endswith(".linear_attn.in_proj_all.weight"):
        key = cfg.linear_heads * cfg.linear_head_dim
        heads = cfg.value_heads
        value = heads * cfg.linear_head_dim
        views = tensor.split(tuple(x // tp for x in (2 * key + value, value, heads, heads)), 0)
        labels = ("in_proj_qkv", "in_proj_z", "in_proj_a", "in_proj_b")
        return {name.replace("in_proj_all", lab): view for lab, view in zip(labels, views)}
    if name.endswith(".self_attn.kv_proj.weight"):
        return dict(zip((name.replace("kv_proj", "k_proj"), name.replace("kv_proj", "v_proj")), tensor.chunk(2, 0)))
    return {name: tensor}


def cast_for_training(model, dtype=torch.bfloat16):
    """Cast to bf16 except the recurrence-sensitive fp32 parameters (A_log, GDN norm, ``keep_fp32`` modules)."""
    keep = {n: p.detach().clone() for n, p in model.named_parameters()
            if n.endswith((".linear_attn.A_log", ".linear_attn.norm.weight"))}
    for mname, module in model.named_modules():
        if getattr(module, "keep_fp32", False):
            keep.update({f"{mname}.{k}" if mname else k: p.detach().clone() for k, p in module.named_parameters()})
    model.to(dtype=dtype)
    for n, p in model.named_parameters():
        if n in keep:
            p.data = keep[n].to(device=p.device, dtype=torch.float32)
    return model
