"""Causal depthwise conv + SiLU kernels (csrc/conv.cu) and the GDN chunk gathers vs fp32 PyTorch."""

import pytest
import torch

from cq_pretrain_b200.ops import _ext
from cq_pretrain_b200.ops import reference as R
from cq_pretrain_b200.ops.gdn_cuda import causal_conv_cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bounds", [(0, 5), (0, 129), (0, 1, 2, 70, 300, 301, 777)])
@pytest.mark.parametrize("C", [64, 1024])
def test_causal_conv_forward_backward(bounds, C):
    assert _ext.has("conv_fwd")
    torch.manual_seed(0)
    n = bounds[-1]
    x = torch.randn(n, C, device="cuda").to(torch.bfloat16)
    w = (torch.rand(C, 4, device="cuda") - 0.5)
    xa, wa = x.clone().requires_grad_(), w.clone().requires_grad_()
    y = causal_conv_cuda(xa, wa, bounds)
    xr, wr = x.float().requires_grad_(), w.clone().requires_grad_()
    ref = R.causal_conv_silu(xr, wr, bounds)
    assert (y.float() - ref).abs().max().item() < 2e-2
    dy = torch.randn(n, C, device="cuda")
    y.backward(dy.to(torch.bfloat16))
    ref.backward(dy.to(torch.bfloat16).float())
    rel_x = (xa.grad.float() - xr.grad).norm() / xr.grad.norm()
    rel_w = (wa.grad.float() - wr.grad).norm() / wr.grad.norm()
    assert rel_x < 1e-2 and rel_w < 1e-2, (rel_x.item(), rel_w.item())


def test_chunk_gather_scatter_roundtrip():
    from cq_pretrain_b200.ops.gdn_cuda import _layout
    torch.manual_seed(1)
    bounds = (0, 10, 140, 141)
    E, H = bounds[-1], 3
    idx, pad, keep, start, count, Nc = _layout(bounds, 64, torch.device("cuda"))
    x = torch.randn(E, H, 128, device="cuda").to(torch.bfloat16)
    ops = _ext.ops()
    out, r = ops.chunk_gather(x, idx, Nc, True, 0.5)
    xf = x.float()
    norm = xf * torch.rsqrt(xf.square().sum(-1, keepdim=True) + 1e-6) * 0.5
    ref = norm.index_select(0, idx.clamp_min(0)).masked_fill(pad[:, None, None], 0)
    ref = ref.view(Nc, 64, H, 128).transpose(1, 2)
    assert (out.float() - ref).abs().max().item() < 1e-2
    back = ops.chunk_scatter(out, keep, x, r, False, 1.0)
    assert torch.equal(back, norm.to(torch.bfloat16))
    # fused L2-norm backward
    dyc = torch.randn(Nc, H, 64, 128, device="cuda")
    dx = ops.chunk_scatter(dyc, keep, x, r, True, 0.5)
    xr = xf.clone().requires_grad_()
    yr = xr * torch.rsqrt(xr.square().sum(-1, keepdim=True) + 1e-6) * 0.5
    dy_events = dyc.transpose(1, 2).reshape(Nc * 64, H, 128).index_select(0, keep)
    yr.backward(dy_events)
    rel = (dx.float() - xr.grad).norm() / xr.grad.norm()
    assert rel < 1e-2, rel.item()


def test_query_conv_matches_torch_path():
    from cq_pretrain_b200.config import tiny_config
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.ops import gdn as GDN
    assert _ext.has("qconv_fwd")
    cfg = tiny_config()
    host, _ = synthetic_batch(cfg, 512, seed=3)
    dp = host.mainline.delta.to("cuda")
    torch.manual_seed(0)
    rows, nc, width, size = host.mainline.rows, len(dp.content_order), 640, 256
    proj = torch.randn(rows, width + 64, device="cuda").to(torch.bfloat16)
    raw = proj[:, :width]                       # strided view, like a split projection
    updates = torch.randn(nc, width, device="cuda").to(torch.bfloat16)
    w = torch.rand(size, 4, device="cuda") - 0.5
    ra, ua, wa = raw.detach().clone().requires_grad_(), updates.clone().requires_grad_(), w.clone().requires_grad_()
    ra_view = torch.cat((ra, proj[:, width:]), 1)[:, :width]   # keep the kernel path on a strided input
    out = GDN.query_conv_silu(ra_view, ua, wa, dp)
    rf, uf, wf = raw.float().requires_grad_(), updates.float().requires_grad_(), w.clone().requires_grad_()
    ref = GDN.query_conv_silu(rf.double(), uf.double(), wf.double(), dp)   # torch path (float64)
    assert (out.double() - ref).abs().max().item() < 2e-2
    dy = torch.randn_like(ref)
    out.backward(dy.to(out.dtype))
    ref.backward(dy)
    for got, want in ((ra.grad, rf.grad), (ua.grad, uf.grad), (wa.grad, wf.grad)):
        rel = (got.double() - want.double()).norm() / want.double().norm()
        assert rel < 1e-2, rel.item()


def test_conv_and_query_node_matches_composed_ops():
    """The fused conv + query conv node (in-place gradient accumulation, disjoint content/query
    rows of d_raw) against the three ops composed in float64."""
    from cq_pretrain_b200.config import tiny_config
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.ops import gdn as GDN
    from cq_pretrain_b200.ops import reference as R
    assert _ext.has("qconv_bwd_into")
    cfg = tiny_config()
    host, _ = synthetic_batch(cfg, 512, seed=5)
    dp = host.mainline.delta.to("cuda")
    torch.manual_seed(1)
    rows, width, size = host.mainline.rows, 768, 256
    proj = torch.randn(rows, width + 64, device="cuda").to(torch.bfloat16)
    w = torch.rand(width, 4, device="cuda") - 0.5
    ra = proj[:, :width].detach().clone().requires_grad_()
    wa = w.clone().requires_grad_()
    ra_view = torch.cat((ra, proj[:, width:]), 1)[:, :width]   # strided rows, like a split projection
    updates, conv, query = GDN.conv_and_query(ra_view, wa, dp, size)
    rf = proj[:, :width].double().requires_grad_()
    wf = w.double().requires_grad_()
    uf = rf.index_select(0, dp.content_order)
    conv_ref = R.causal_conv_silu(uf, wf, dp.content_bounds)
    query_ref = GDN.query_conv_silu(rf, uf, wf[:size], dp)
    assert (updates.double() - uf).abs().max().item() == 0
    for got, want in ((conv, conv_ref), (query, query_ref)):
        assert (got.double() - want).abs().max().item() < 2e-2
    dc, dq = torch.randn_like(conv_ref), torch.randn_like(query_ref)
    torch.autograd.backward((conv, query), (dc.to(conv.dtype), dq.to(query.dtype)))
    torch.autograd.backward((conv_ref, query_ref), (dc, dq))
    for got, want in ((ra.grad, rf.grad), (wa.grad, wf.grad)):
        rel = (got.double() - want).norm() / want.norm()
        assert rel < 1e-2, rel.item()
