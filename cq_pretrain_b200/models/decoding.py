"""Request-local CQ text decoding with committed-content caches (TP = 1).

Prefill runs the ordinary CQ plan of one document whose last content position is the
placeholder of the first unknown token; that placeholder is *not* committed (its GDN write
event becomes read-only, and its attention key is dropped). Each ``advance(token)`` then runs
two rows through every layer: the sampled token as content (appends its KV, updates the fp32
GDN state and the conv history) and a fresh text-mask query that reads the committed prefix
(reference ``models/decoding.py:16-171``). No dense mask is ever built.

``GraphedCQDecoder`` (CUDA) replays the per-token step as one CUDA graph: the KV caches become
fixed-capacity buffers with a device-side key count, the conv history and GDN state are updated
in place, and the token and position are read from device tensors, so every step after the first
(eager, which also warms up the kernels) is a single graph launch.
"""

from __future__ import annotations

from dataclasses import replace

import torch
import torch.nn.functional as F

from ..data.plan import mrope_tables
from ..ops import gdn as GDN
from ..ops import reference as R


def _delta_step(layer, x, cache):
    cfg = layer.cfg
    hk, h, d = cfg.linear_heads, cfg.value_heads, cfg.linear_head_dim
    size = hk * d
    raw, z, a, b = layer.project(x)           # rows: [content, query]
    weight = layer.conv1d.weight[:, 0].to(raw.dtype)
    history = cache["conv"]                   # [K-1, C] raw committed inputs (oldest first)
    conv = raw[0] * weight[:, -1]
    for j in range(history.shape[0]):
        conv = conv + history[j] * weight[:, j]
    conv = F.silu(conv.float()).to(raw.dtype) if raw.dtype != torch.float64 else F.silu(conv)
    if history.shape[0]:
        history.copy_(torch.cat((history[1:], raw[:1])))   # the query's history includes the new token
    query = raw[1, :size] * weight[:size, -1]
    for j in range(history.shape[0]):
        query = query + history[j, :size] * weight[:size, j]
    query = F.silu(query.float()).to(raw.dtype) if raw.dtype != torch.float64 else F.silu(query)
    cq, k, v = conv.split((size, size, h * d), -1)
    q = torch.stack((cq, query)).reshape(2, hk, d)
    k = k.reshape(1, hk, d)
    v = v.reshape(1, h, d)
    if h != hk:
        q, k = (t.repeat_interleave(h // hk, dim=1) for t in (q, k))
    ctrl = torch.float64 if x.dtype == torch.float64 else torch.float32
    g = -layer.A_log.to(ctrl).exp() * F.softplus(a[:1].to(ctrl) + layer.dt_bias.to(ctrl))
    beta = b[:1].to(ctrl).sigmoid()
    # fused recurrent step on the cached fp32 state [H, Dk, Dv] (in place; one kernel on CUDA)
    y = GDN.decode_step(cache["state"][0], q, k[0], v[0], g[0], beta[0]).to(x.dtype)
    return layer.out_proj(layer.norm(y, z.reshape(2, h, d)).flatten(-2))


def _attention_step(layer, x, rope, cache):
    cfg = layer.cfg
    q, gate = layer.q_proj(x).reshape(2, cfg.heads, 2 * cfg.head_dim).chunk(2, -1)
    q = layer.q_norm(q)
    if cfg.qwen_fused_projections:
        k, v = (t.reshape(1, cfg.kv_heads, cfg.head_dim) for t in layer.kv_proj(x[:1]).chunk(2, -1))
    else:
        k = layer.k_proj(x[:1]).reshape(1, cfg.kv_heads, cfg.head_dim)
        v = layer.v_proj(x[:1]).reshape(1, cfg.kv_heads, cfg.head_dim)
    k = layer.k_norm(k)
    cos, sin = rope
    q = R.rotary_half(q, cos, sin, cfg.rotary_dim)
    k = R.rotary_half(k, cos[:1], sin[:1], cfg.rotary_dim)
    cache["k"] = torch.cat((cache["k"], k))
    cache["v"] = torch.cat((cache["v"], v.contiguous()))
    n = cache["k"].shape[0]
    # the content row sees the committed prefix including itself; so does the next query
    y = R.range_attention(q, cache["k"], cache["v"], torch.zeros(2, dtype=torch.int32, device=x.device),
                          torch.full((2,), n, dtype=torch.int32, device=x.device))
    return layer.o_proj((y * gate.sigmoid()).flatten(-2))


def _attention_step_static(layer, x, rope, cache, count, starts):
    """``_attention_step`` over fixed-capacity KV buffers: the content row's K / V land at row
    ``count`` and both rows read keys ``[0, count + 1)`` (device tensors, no host sync)."""
    from ..ops import attention as ATT
    cfg = layer.cfg
    q, gate = layer.q_proj(x).reshape(2, cfg.heads, 2 * cfg.head_dim).chunk(2, -1)
    q = layer.q_norm(q)
    if cfg.qwen_fused_projections:
        k, v = (t.reshape(1, cfg.kv_heads, cfg.head_dim) for t in layer.kv_proj(x[:1]).chunk(2, -1))
    else:
        k = layer.k_proj(x[:1]).reshape(1, cfg.kv_heads, cfg.head_dim)
        v = layer.v_proj(x[:1]).reshape(1, cfg.kv_heads, cfg.head_dim)
    k = layer.k_norm(k)
    cos, sin = rope
    q = R.rotary_half(q, cos, sin, cfg.rotary_dim)
    k = R.rotary_half(k, cos[:1], sin[:1], cfg.rotary_dim)
    index = count.long()
    cache["k_buf"].index_copy_(0, index, k.to(cache["k_buf"].dtype))
    cache["v_buf"].index_copy_(0, index, v.to(cache["v_buf"].dtype))
    ends = (count + 1).expand(2).contiguous()
    y = ATT.cq_attention(q.contiguous(), cache["k_buf"], cache["v_buf"], starts, ends)
    return layer.o_proj((y * gate.sigmoid()).flatten(-2))


class CQDecoder:
    """Prefill once, then ``advance(token)`` per sampled token; ``hidden`` is the query readout."""

    @torch.no_grad()
    def __init__(self, model, batch, max_new_tokens):
        cfg = model.cfg
        plan = batch.mainline
        s = plan.content_length
        if (cfg.method != "CQ_IT" or plan.queries != 1 or int(plan.query_positions[0]) != s - 1
                or bool(plan.query_image.any()) or int(batch.segments.min()) < 0
                or len(torch.unique(batch.segments)) != 1):
            raise ValueError("CQ decoding needs one document whose only query reads its final placeholder")
        self.model, self.limit, self.step = model, max_new_tokens, 0
        device = model.embedding.weight.device
        delta = plan.delta
        writes = delta.event_write.clone()
        last = len(delta.content_order) - 1
        writes[writes == last] = len(delta.content_order)   # placeholder: read-only
        local = replace(batch, mainline=replace(plan, delta=replace(delta, event_write=writes)))
        local = local.to(device)
        self.caches = [dict() for _ in model.layers]
        output = model.backbone(local, cache=self.caches)
        for layer, cache in zip(model.layers, self.caches):
            if hasattr(layer, "self_attn"):
                cache["k"], cache["v"] = cache["k"][: s - 1], cache["v"][: s - 1]
        self.hidden = output.index_select(0, local.mainline.output_positions.to(device))
        base = plan.query_rope.double()
        steps = torch.arange(max_new_tokens + 1, dtype=torch.float64)
        positions = base + steps[None]
        cos, sin = mrope_tables(positions, cfg)
        dtype = model.embedding.weight.dtype
        self.rope = (cos.to(device=device, dtype=dtype), sin.to(device=device, dtype=dtype))
        self.ids = torch.tensor([0, cfg.text_mask_token_id], device=device)

    @torch.no_grad()
    def advance(self, token):
        if self.step >= self.limit:
            raise ValueError("CQ decode capacity exceeded")
        model = self.model
        self.ids[0] = int(token)
        hidden = model.embedding.partial(self.ids)
        rope = tuple(t[self.step:self.step + 2] for t in self.rope)
        for layer, cache in zip(model.layers, self.caches):
            normed = layer.input_layernorm(hidden)
            if hasattr(layer, "linear_attn"):
                mixed = _delta_step(layer.linear_attn, normed, cache)
            else:
                mixed = _attention_step(layer.self_attn, normed, rope, cache)
            hidden = hidden + mixed
            hidden = hidden + layer.mlp(layer.post_attention_layernorm(hidden))
        self.step += 1
        self.hidden = model.final_norm(hidden[1:2])
        return self.hidden


class GraphedCQDecoder(CQDecoder):
    """``CQDecoder`` whose step after the first is one CUDA-graph replay (CUDA tensors only).

    Capacity is fixed at construction: the KV buffers hold the committed prefix plus
    ``max_new_tokens``. ``advance`` copies the token into a device tensor, replays the graph and
    returns the (static) query readout; the returned tensor is overwritten by the next call.
    """

    @torch.no_grad()
    def __init__(self, model, batch, max_new_tokens):
        super().__init__(model, batch, max_new_tokens)
        device = model.embedding.weight.device
        if device.type != "cuda":
            raise ValueError("graph replay needs a CUDA model")
        committed = None
        for layer, cache in zip(model.layers, self.caches):
            if hasattr(layer, "self_attn"):
                k, v = cache.pop("k"), cache.pop("v")
                committed = k.shape[0]
                for name, t in (("k_buf", k), ("v_buf", v)):
                    buf = t.new_zeros((committed + max_new_tokens + 1,) + tuple(t.shape[1:]))
                    buf[:committed] = t
                    cache[name] = buf
        self.count = torch.tensor([committed or 0], dtype=torch.int32, device=device)
        self.starts = torch.zeros(2, dtype=torch.int32, device=device)
        self.position = torch.zeros(1, dtype=torch.long, device=device)
        self.pair = torch.arange(2, device=device)
        self.token = torch.zeros(1, dtype=torch.long).pin_memory()
        self.copied = torch.cuda.Event()          # the pinned token buffer may be rewritten after it
        self.graph, self.out = None, None

    def _step(self):
        model = self.model
        hidden = model.embedding.partial(self.ids)
        rows = self.position + self.pair
        rope = tuple(t.index_select(0, rows) for t in self.rope)
        for layer, cache in zip(model.layers, self.caches):
            normed = layer.input_layernorm(hidden)
            if hasattr(layer, "linear_attn"):
                mixed = _delta_step(layer.linear_attn, normed, cache)
            else:
                mixed = _attention_step_static(layer.self_attn, normed, rope, cache, self.count, self.starts)
            hidden = hidden + mixed
            hidden = hidden + layer.mlp(layer.post_attention_layernorm(hidden))
        self.count += 1
        self.position += 1
        return model.final_norm(hidden[1:2])

    @torch.no_grad()
    def advance(self, token):
        if self.step >= self.limit:
            raise ValueError("CQ decode capacity exceeded")
        self.copied.synchronize()
        self.token[0] = int(token)
        self.ids[:1].copy_(self.token, non_blocking=True)
        self.copied.record()
        if self.step == 0:
            self.hidden = self._step()             # eager: also loads every kernel once
        else:
            if self.graph is None:
                self.graph = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side):
                    self.out = self._step()        # recorded only; replayed below
                torch.cuda.current_stream().wait_stream(side)
            self.graph.replay()
            self.hidden = self.out
        self.step += 1
        return self.hidden
