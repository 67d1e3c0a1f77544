"""Wan2.1 DiT renderer conditioned on CQ visual-query hidden states, trained by flow matching.

Architecture (reference ``models/generator_wan21.py:18-297``): patch embedding (Conv3d 1x2x2 run as
a GEMM), FP32 time embedding and 6-way adaLN modulation, blocks of [modulated LN -> self
attention with full-width Q/K RMSNorm and 3D RoPE -> fp32 gated residual -> LN -> cross
attention over the projected conditions -> modulated LN -> GELU-tanh FFN -> fp32 gated
residual], and a modulated head. The adapter ``text_embedding`` maps backbone width ->
1536 -> 1536 with GELU.

Sequence parallel: DiT tokens are row-sharded across TP between modules. Self-attention's q and
kv projections share one in-kernel all-gather of the rows; the cross-attention context is
gathered once per DiT call and read by every block's kv projection. The full-width Q/K RMSNorm
needs the sum of squares over all heads, which live on different TP ranks: on CUDA one kernel per
call exchanges the per-row partial sums over NVLink peer memory (no NCCL call).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import attention as ATT
from ..ops import norms as N
from ..ops import rope as ROPE
from ..parallel import layers as PL
from ..parallel import state as ps


class FP32Linear(nn.Linear):
    keep_fp32 = True

    def forward(self, x):
        return F.linear(x.float(), self.weight.float(), self.bias.float())


class WanRMSNorm(nn.Module):
    """RMSNorm over the whole projected width, whose heads are spread over TP ranks."""

    def __init__(self, width, eps):
        super().__init__()
        self.eps = eps
        self.weight = PL.mark_sharded(nn.Parameter(torch.ones(width // ps.tp_size())))

    def forward(self, x):
        if ps.tp_size() > 1:
            from ..parallel import symmetric
            ws = symmetric.workspace()
            if ws is not None and ws.supports_rms(x):
                # in-kernel exchange of the per-row sums of squares over NVLink (no NCCL call)
                return _TPRMSNorm.apply(x, self.weight, ws, x.shape[-1] * ps.tp_size(), self.eps)
        elif x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
            # one kernel each way: the (1 + w) RMSNorm with w - 1 gives x r w
            return N.rms_norm(x.contiguous(), self.weight - 1, self.eps)
        sq = x.float().square().sum(-1, keepdim=True)
        if ps.tp_size() > 1:
            sq = PL.sum_tp(sq)     # every rank normalises its own heads with the full-width sum
        variance = sq / (x.shape[-1] * ps.tp_size())
        return (x.float() * torch.rsqrt(variance + self.eps)).to(x.dtype) * self.weight.to(x.dtype)


class _TPRMSNorm(torch.autograd.Function):
    """RMSNorm over a width split across TP ranks; both passes exchange per-row sums in-kernel."""

    @staticmethod
    def forward(ctx, x, weight, ws, total_dim, eps):
        w = weight.float().contiguous()
        y, rstd = ws.rms_forward(x, w, total_dim, eps)
        ctx.save_for_backward(x, w, rstd)
        ctx.ws, ctx.total_dim, ctx.wdtype = ws, total_dim, weight.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = ctx.ws.rms_backward(dy.to(torch.bfloat16), x, w, rstd, ctx.total_dim)
        return dx, dw.to(ctx.wdtype), None, None, None


class Attention(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        dim = cfg.dit_width
        self.heads = cfg.dit_heads // ps.tp_size()
        self.head_dim = dim // cfg.dit_heads
        self.q = PL.ColumnLinear(dim, dim, bias=True)
        self.kv = PL.ColumnLinear(dim, 2 * dim, bias=True, stride=2)
        self.o = PL.RowLinear(dim, dim, bias=True)
        self.norm_q = WanRMSNorm(dim, cfg.norm_eps)
        self.norm_k = WanRMSNorm(dim, cfg.norm_eps)

    def _fused_qk(self, q, k, layout):
        """Self-attention q / k through one kernel each way: the full-width RMSNorm of both (per-row
        sums exchanged over NVLink in-kernel at TP > 1) and the complex-pair RoPE. None where the
        kernel does not apply (CPU, or TP > 1 without the peer workspace)."""
        if not N.qk_norm_rope_supported(q, k):
            return None
        exchange = None
        if ps.tp_size() > 1:
            from ..parallel import symmetric
            ws = symmetric.workspace()
            if ws is None or not ws.supports_qk(q, k):
                return None
            exchange = ws.exchange_kwargs
        total = q.shape[-1] * ps.tp_size()
        qo, ko = N.qk_norm_rope(q, k, self.norm_q.weight, self.norm_k.weight, layout.cos_rows, layout.sin_rows,
                                self.head_dim, total, self.norm_q.eps, exchange)
        return qo.view(-1, self.heads, self.head_dim), ko.view(-1, self.heads, self.head_dim)

    def project_kv(self, context_full):
        k, v = self.kv(context_full, gathered=True).chunk(2, -1)
        k = self.norm_k(k).reshape(-1, self.heads, self.head_dim)
        return k, v.reshape(-1, self.heads, self.head_dim)

    def forward(self, x, layout, context=None, cached_kv=None):
        """``x``: this rank's rows; ``context``: every rank's condition rows (gathered once per call)."""
        if context is None and cached_kv is None:
            q, kv = PL.column_pair(x, self.q, self.kv)
            k, v = kv.chunk(2, -1)
            v = v.reshape(-1, self.heads, self.head_dim)
            fused = self._fused_qk(q, k, layout)
            if fused is not None:
                q, k = fused
                y = ATT.varlen_attention(q, k, v, layout.row_ends, layout.row_ends, ranges=layout.self_ranges)
                return self.o(y.flatten(1))
            k = self.norm_k(k).reshape(-1, self.heads, self.head_dim)
        else:
            q = self.q(x)
            k, v = cached_kv if cached_kv is not None else self.project_kv(context)
        q = self.norm_q(q).reshape(-1, self.heads, self.head_dim)
        if context is None and cached_kv is None:
            q = ROPE.rotary_pairs(q, layout.cos_rows, layout.sin_rows)
            k = ROPE.rotary_pairs(k, layout.cos_rows, layout.sin_rows)
            y = ATT.varlen_attention(q, k, v, layout.row_ends, layout.row_ends, ranges=layout.self_ranges)
        else:
            y = ATT.varlen_attention(q, k, v, layout.row_ends, layout.cond_ends, ranges=layout.cross_ranges)
        return self.o(y.flatten(1))


_ONES: dict = {}


def _ones(width, device):
    """A cached fp32 ``[1, width]`` ones row (the gate of an ungated residual add)."""
    key = (width, str(device))
    if key not in _ONES:
        _ONES[key] = torch.ones(1, width, device=device)
    return _ONES[key]


class Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        dim = cfg.dit_width
        self.eps = cfg.norm_eps
        self.self_attn = Attention(cfg)
        self.norm3 = nn.LayerNorm(dim, eps=cfg.norm_eps)
        self.cross_attn = Attention(cfg)
        self.ffn = nn.Sequential(PL.ColumnLinear(dim, cfg.dit_ffn, bias=True), nn.GELU(approximate="tanh"),
                                 PL.RowLinear(cfg.dit_ffn, dim, bias=True))
        self.modulation = nn.Parameter(torch.randn(1, 6, dim) / math.sqrt(dim))

    def forward(self, x, modulation, context, layout, cached_kv=None):
        # modulation: [targets, 6, dim] fp32; layout.local_sample maps local rows -> target
        mod = modulation + self.modulation.float()
        shift, scale, gate, fshift, fscale, fgate = mod.unbind(1)
        idx = layout.local_sample
        dtype = self.self_attn.q.weight.dtype
        y = self.self_attn(N.layer_norm_modulate(x, scale, shift, self.eps, idx).to(dtype), layout)
        x = N.gated_add(x.float(), y, gate, idx)
        # norm3 (affine LayerNorm) as the modulated-LN kernel with one modulation row: scale = w - 1,
        # shift = b (their gradients are the kernel's modulation gradients)
        zeros = layout.zero_rows if x.is_cuda else None
        normed = N.layer_norm_modulate(x, (self.norm3.weight.float() - 1)[None], self.norm3.bias.float()[None],
                                       self.eps, zeros)
        cross = self.cross_attn(normed.to(y.dtype), layout, context, cached_kv)
        x = N.gated_add(x, cross, _ones(x.shape[-1], x.device), zeros) if x.is_cuda else x + cross.float()
        h = N.layer_norm_modulate(x, fscale, fshift, self.eps, idx).to(y.dtype)
        h = self.ffn[2](self.ffn[1](self.ffn[0](h)))
        return N.gated_add(x, h, fgate, idx)


class Head(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        dim = cfg.dit_width
        self.eps = cfg.norm_eps
        self.modulation = nn.Parameter(torch.randn(1, 2, dim) / math.sqrt(dim))
        self.head = nn.Linear(dim, cfg.latent_channels * 4)

    def forward(self, x, time, idx):
        shift, scale = (time[:, None].float() + self.modulation.float()).unbind(1)
        h = N.layer_norm_modulate(x, scale, shift, self.eps, idx).to(self.head.weight.dtype)
        value = F.linear(h, self.head.weight, self.head.bias)
        # the native head emits [ph, pw, C]; patches are stored [C, ph, pw]
        return value.reshape(-1, 2, 2, value.shape[-1] // 4).permute(0, 3, 1, 2).flatten(1)


class PatchEmbedding(nn.Module):
    """Conv3d (1x2x2) weights executed as a GEMM over patchified latents."""

    def __init__(self, cfg):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(cfg.dit_width, cfg.latent_channels, 1, 2, 2))
        self.bias = nn.Parameter(torch.zeros(cfg.dit_width))
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))

    def forward(self, patches):
        return F.linear(patches.to(self.weight.dtype), self.weight.flatten(1), self.bias)


class RowLayout:
    """Device-side row geometry of one DiT call, padded so rows divide evenly across TP."""

    def __init__(self, gen, device, tp, tp_rank, pad_to=None):
        pad_to = pad_to or (128 if tp > 1 else 8)   # 128-row blocks per rank enable the fused TP kernels
        lengths = list(gen.lengths)
        total = sum(lengths)
        unit = tp * pad_to
        padded = -(-total // unit) * unit
        self.pad = padded - total
        self.rows = padded
        ends = [int(e) for e in gen.video_ends]
        if self.pad:
            ends.append(padded)  # padding rows form their own sample (zero loss weight)
        self.row_ends = tuple(ends)
        cond = [int(e) for e in gen.text_ends]
        if self.pad:
            cond.append(cond[-1])  # padding sample reads no conditions
        self.cond_ends = tuple(cond)
        sample = gen.video_sample_indices
        if self.pad:
            sample = torch.cat((sample, sample.new_zeros(self.pad)))
        self.sample = sample.to(device)
        n = padded // tp
        self.local_sample = self.sample[tp_rank * n:(tp_rank + 1) * n]
        # every local row -> modulation row 0, and an all-ones gate: the affine norm3 and the
        # ungated cross-attention residual reuse the modulation / gated-add kernels
        self.zero_rows = torch.zeros(n, dtype=torch.int32, device=device)
        cos, sin = gen.cos, gen.sin
        if self.pad:
            cos = torch.cat((cos, cos.new_ones(self.pad, cos.shape[1])))
            sin = torch.cat((sin, sin.new_zeros(self.pad, sin.shape[1])))
        self.cos_rows, self.sin_rows = cos.to(device), sin.to(device)
        self.self_ranges = ATT.ranges_from_ends(self.row_ends, self.row_ends, device) if device.type == "cuda" else None
        self.cross_ranges = ATT.ranges_from_ends(self.row_ends, self.cond_ends, device) if device.type == "cuda" else None


_ROW_LAYOUTS: dict = {}


def row_layout(gen, device, tp, tp_rank):
    """The ``RowLayout`` of a DiT call, cached per geometry: every tensor in it (sample of each
    row, RoPE rows, attention ranges) is a function of the targets' grids, lengths and condition
    counts, so a repeated geometry reuses the device tensors instead of copying them again (and a
    CUDA-graph capture finds them already on the device)."""
    key = (gen.grids, gen.lengths, gen.query_counts, gen.video_ends, gen.text_ends, tuple(gen.cos.shape),
           str(gen.cos.dtype), tp, tp_rank, str(device))
    hit = _ROW_LAYOUTS.get(key)
    if hit is None:
        if len(_ROW_LAYOUTS) > 32:
            _ROW_LAYOUTS.clear()
        hit = _ROW_LAYOUTS[key] = RowLayout(gen, device, tp, tp_rank)
    return hit


class Wan21Generator(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        dim = cfg.dit_width
        self.patch_embedding = PatchEmbedding(cfg)
        self.text_embedding = nn.Sequential(PL.ColumnLinear(cfg.width, dim, bias=True), nn.GELU(approximate="tanh"),
                                            PL.RowLinear(dim, dim, bias=True))
        self.time_embedding = nn.Sequential(FP32Linear(cfg.wan_freq_dim, dim), nn.SiLU(), FP32Linear(dim, dim))
        self.time_projection = nn.Sequential(nn.SiLU(), FP32Linear(dim, 6 * dim))
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.dit_layers)])
        self.head = Head(cfg)

    def project_conditions(self, conditions, gen):
        """conditions ``[targets, max_q, width]`` (replicated) -> row-sharded ``[sum q (padded), dit]``."""
        ctx = conditions.reshape(-1, self.cfg.width).index_select(0, gen.condition_indices.to(conditions.device))
        tp = ps.tp_size()
        pad = (-ctx.shape[0]) % ((128 if tp > 1 else 8) * tp)
        if pad:
            ctx = torch.cat((ctx, ctx.new_zeros(pad, ctx.shape[1])))
        ctx = PL.split_rows(ctx)
        h = self.text_embedding[0](ctx.to(self.text_embedding[0].weight.dtype))
        return self.text_embedding[2](self.text_embedding[1](h))

    @torch.no_grad()
    def cache_condition_kv(self, context):
        ctx = PL.gather_rows(context) if ps.tp_size() > 1 else context
        return tuple(tuple(t.contiguous() for t in block.cross_attn.project_kv(ctx)) for block in self.blocks)

    @staticmethod
    def gather_context(context):
        """All ranks' projected condition rows: one all-gather per DiT call, read by every block."""
        return PL.gather_rows(context) if ps.tp_size() > 1 else context

    def predict(self, xt, conditions, gen, projected=None, cached_kv=None):
        """Velocity prediction for packed noisy patches ``xt [sum L, C*4]`` (all rows, every rank)."""
        out, layout = self.predict_local(xt, conditions, gen, projected, cached_kv)
        out = PL.gather_rows(out) if ps.tp_size() > 1 else out
        return out[: out.shape[0] - layout.pad]

    def predict_local(self, xt, conditions, gen, projected=None, cached_kv=None):
        """This rank's row shard of the prediction (fp32) and the row layout."""
        st = ps.state()
        device = xt.device
        layout = row_layout(gen, device, st.tp, st.tp_rank)
        time = self.time_embedding(gen.time_features.float().to(device))
        e = self.time_projection(time).reshape(-1, 6, self.cfg.dit_width)
        context = self.project_conditions(conditions, gen) if projected is None else projected
        context = self.gather_context(context) if cached_kv is None else None
        if layout.pad:
            xt = torch.cat((xt, xt.new_zeros(layout.pad, xt.shape[1])))
        x = self.patch_embedding(PL.split_rows(xt) if st.tp > 1 else xt)
        recompute = self.training and torch.is_grad_enabled()
        for i, block in enumerate(self.blocks):
            kv = None if cached_kv is None else cached_kv[i]
            if recompute and (self.cfg.checkpoint_dit or i >= self.cfg.dit_layers - self.cfg.checkpoint_dit_layers):
                x = torch.utils.checkpoint.checkpoint(block, x, e, context, layout, kv, use_reentrant=False)
            else:
                x = block(x, e, context, layout, kv)
        return self.head(x, time, layout.local_sample).float(), layout

    def forward(self, conditions, batch):
        """Flow-matching loss ``sum_i w_i mean_c (v_hat - (eps - x0))^2`` with ``xt = (1-s) x0 + s eps``."""
        gen = batch.generation
        sigma = batch.times.index_select(0, gen.video_sample_indices.to(batch.times.device))[:, None].float()
        x0, eps = batch.latents.float(), batch.noise.float()
        xt = (1 - sigma) * x0 + sigma * eps
        local, layout = self.predict_local(xt, conditions, gen)
        target = eps - x0
        weights = gen.loss_weights.to(local.device)
        if layout.pad:
            target = torch.cat((target, target.new_zeros(layout.pad, target.shape[1])))
            weights = torch.cat((weights, weights.new_zeros(layout.pad)))
        lo, hi = PL.local_row_range(layout.rows)
        error = (local - target[lo:hi]).square().mean(-1)
        loss = (error * weights[lo:hi]).sum()
        return PL.reduce_tp(loss) if ps.tp_size() > 1 else loss
