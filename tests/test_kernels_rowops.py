"""sm_100a row kernels vs plain-PyTorch fp32 references (forward and backward)."""

import pytest
import torch
import torch.nn.functional as F

from cq_pretrain_b200.ops import _ext, activation, norms
from cq_pretrain_b200.ops import reference as R

pytestmark = pytest.mark.gpu


def _grads(fn, *inputs):
    out = fn(*inputs)
    g = torch.randn_like(out.float()).to(out.dtype)
    grads = torch.autograd.grad(out, inputs, g, allow_unused=True)
    return out, grads


@pytest.mark.parametrize("width", [128, 256, 1536, 2048])
def test_rms_norm(width):
    assert _ext.has("rms_norm_fwd")
    torch.manual_seed(0)
    x = torch.randn(1000, width, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (0.1 * torch.randn(width, device="cuda")).to(torch.bfloat16).requires_grad_()
    g = torch.randn(1000, width, device="cuda", dtype=torch.bfloat16)
    y = norms.rms_norm(x, w, 1e-6)
    dx, dw = torch.autograd.grad(y, (x, w), g)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = R.rms_norm(xr, wr, 1e-6)
    dxr, dwr = torch.autograd.grad(yr, (xr, wr), g.float())
    torch.testing.assert_close(y.float(), yr, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(dx.float(), dxr, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(dw.float(), dwr, atol=0.5, rtol=2e-2)


def test_gated_norm():
    torch.manual_seed(1)
    x = torch.randn(4096, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    z = torch.randn(4096, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(128, device="cuda")).requires_grad_()
    g = torch.randn(4096, 128, device="cuda", dtype=torch.bfloat16)
    y = norms.gated_rms_norm(x, z, w, 1e-6)
    dx, dz, dw = torch.autograd.grad(y, (x, z, w), g)
    xr, zr, wr = (t.detach().float().requires_grad_() for t in (x, z, w))
    yr = (xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + 1e-6)) * wr * F.silu(zr)
    dxr, dzr, dwr = torch.autograd.grad(yr, (xr, zr, wr), g.float())
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(dx.float(), dxr, atol=5e-2, rtol=5e-2)
    torch.testing.assert_close(dz.float(), dzr, atol=5e-2, rtol=5e-2)
    torch.testing.assert_close(dw, dwr, atol=1.0, rtol=3e-2)


@pytest.mark.parametrize("xdtype", [torch.float32, torch.bfloat16])
def test_layer_norm_modulate(xdtype):
    torch.manual_seed(2)
    rows, width = 3000, 1536
    x = torch.randn(rows, width, device="cuda", dtype=xdtype, requires_grad=True)
    scale = (0.1 * torch.randn(3, width, device="cuda")).requires_grad_()
    shift = (0.1 * torch.randn(3, width, device="cuda")).requires_grad_()
    idx = torch.cat([torch.full((n,), i, device="cuda") for i, n in enumerate((1000, 1500, 500))])
    g = torch.randn(rows, width, device="cuda", dtype=torch.bfloat16)
    y = norms.layer_norm_modulate(x, scale, shift, 1e-6, idx)
    grads = torch.autograd.grad(y, (x, scale, shift), g)
    xr, sr, hr = (t.detach().float().requires_grad_() for t in (x, scale, shift))
    yr = R.layer_norm_modulate(xr, sr[idx], hr[idx], 1e-6)
    ref = torch.autograd.grad(yr, (xr, sr, hr), g.float())
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=2e-2)
    for a, b in zip(grads, ref):
        torch.testing.assert_close(a.float(), b, atol=0.2, rtol=2e-2)


def test_gated_add():
    torch.manual_seed(3)
    rows, width = 2048, 1536
    x = torch.randn(rows, width, device="cuda", requires_grad=True)
    b = torch.randn(rows, width, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    gate = torch.randn(2, width, device="cuda", requires_grad=True)
    idx = (torch.arange(rows, device="cuda") >= 700).long()
    g = torch.randn(rows, width, device="cuda")
    y = norms.gated_add(x, b, gate, idx)
    grads = torch.autograd.grad(y, (x, b, gate), g)
    xr, br, gr = (t.detach().float().requires_grad_() for t in (x, b, gate))
    yr = xr + gr[idx] * br
    ref = torch.autograd.grad(yr, (xr, br, gr), g)
    torch.testing.assert_close(y, yr, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(grads[0], ref[0])
    torch.testing.assert_close(grads[1].float(), ref[1], atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(grads[2], ref[2], atol=1e-2, rtol=1e-4)


def test_swiglu():
    torch.manual_seed(4)
    x = torch.randn(1500, 2 * 6144, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = torch.randn(1500, 6144, device="cuda", dtype=torch.bfloat16)
    y = activation.swiglu(x)
    (dx,) = torch.autograd.grad(y, (x,), g)
    xr = x.detach().float().requires_grad_()
    a, u = xr.chunk(2, -1)
    yr = F.silu(a) * u
    (dxr,) = torch.autograd.grad(yr, (xr,), g.float())
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(dx.float(), dxr, atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("rows,cols", [(2048, 1536), (77, 40), (1, 8)])
def test_column_sum(rows, cols):
    torch.manual_seed(5)
    x = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
    got = _ext.ops().column_sum(x)
    torch.testing.assert_close(got, x.float().sum(0), atol=1e-3, rtol=1e-4)
    again = _ext.ops().column_sum(x)
    assert torch.equal(got, again)   # fixed reduction order


def test_rope_pairs_matches_reference():
    from cq_pretrain_b200.ops import rope
    torch.manual_seed(6)
    x = torch.randn(300, 12, 128, device="cuda").to(torch.bfloat16).requires_grad_()
    ang = torch.rand(300, 64, device="cuda") * 6
    y = rope.rotary_pairs(x, ang.cos(), ang.sin())
    xr = x.detach().float().requires_grad_()
    yr = R.rotary_pairs(xr, ang.cos(), ang.sin())
    torch.testing.assert_close(y.float(), yr, atol=2e-2, rtol=1e-2)
    g = torch.randn_like(yr)
    y.backward(g.to(y.dtype))
    yr.backward(g)
    torch.testing.assert_close(x.grad.float(), xr.grad, atol=3e-2, rtol=2e-2)


def test_wan_rmsnorm_tp1_kernel_matches_torch():
    from cq_pretrain_b200.models.wan21 import WanRMSNorm
    torch.manual_seed(7)
    norm = WanRMSNorm(1536, 1e-6).cuda()
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn_like(norm.weight))
    x = torch.randn(500, 1536, device="cuda").to(torch.bfloat16).requires_grad_()
    y = norm(x)
    xr, wr = x.detach().float().requires_grad_(), norm.weight.detach().clone().requires_grad_()
    yr = xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + 1e-6) * wr
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=2e-2)
    g = torch.randn_like(yr)
    y.backward(g.to(y.dtype))
    yr.backward(g)
    torch.testing.assert_close(x.grad.float(), xr.grad, atol=5e-2, rtol=3e-2)
    rel = (norm.weight.grad - wr.grad).norm() / wr.grad.norm()
    assert rel < 2e-2


def test_rms_norm_residual_fuses_the_residual_gradient():
    """``(x, norm(x))`` with both outputs used: the input gradient (residual + norm paths, summed in
    the norm's backward kernel) and the weight gradient match fp32 autograd."""
    torch.manual_seed(3)
    x = torch.randn(1000, 2048, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(2048, device="cuda") * 0.1).requires_grad_()
    res, y = norms.rms_norm_residual(x, w, 1e-6)
    assert res.data_ptr() == x.data_ptr()
    g_res, g_y = torch.randn_like(res), torch.randn_like(y)
    (res.float() * g_res.float()).sum().add_((y.float() * g_y.float()).sum()).backward()
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = R.rms_norm(xr, wr, 1e-6)
    (xr * g_res.float()).sum().add_((yr * g_y.float()).sum()).backward()
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=3e-2)
    assert ((x.grad.float() - xr.grad).norm() / xr.grad.norm()).item() < 1e-2
    assert ((w.grad.float() - wr.grad).norm() / wr.grad.norm()).item() < 1e-2


def test_gated_norm_reads_strided_gate_in_place():
    """The GDN output norm with the gate read in place from a wider projection row ([tokens, heads,
    128] with a token stride) matches the fp32 reference, gradients included."""
    from cq_pretrain_b200.ops import norms as N
    torch.manual_seed(5)
    tokens, heads = 777, 16
    proj = torch.randn(tokens, heads * 128 + 96, device="cuda").to(torch.bfloat16)
    z = proj[:, 64:64 + heads * 128].reshape(tokens, heads, 128)
    x = torch.randn(tokens, heads, 128, device="cuda").to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(128, device="cuda")).to(torch.bfloat16)
    xa, za, wa = x.clone().requires_grad_(), z.detach().clone(), w.clone().requires_grad_()
    pa = proj.clone().requires_grad_()
    zv = pa[:, 64:64 + heads * 128].reshape(tokens, heads, 128)
    assert zv.stride(0) == heads * 128 + 96
    y = N.gated_rms_norm(xa, zv, wa, 1e-6)
    xr, zr, wr = x.float().requires_grad_(), za.float().requires_grad_(), w.float().requires_grad_()
    yr = xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + 1e-6) * wr * torch.nn.functional.silu(zr)
    assert ((y.float() - yr).norm() / yr.norm()).item() < 1e-2
    g = torch.randn_like(yr)
    y.backward(g.to(y.dtype))
    yr.backward(g)
    dz = pa.grad[:, 64:64 + heads * 128].reshape(tokens, heads, 128).float()
    assert pa.grad[:, :64].abs().max().item() == 0 and pa.grad[:, 64 + heads * 128:].abs().max().item() == 0
    for got, want in ((xa.grad.float(), xr.grad), (dz, zr.grad), (wa.grad.float(), wr.grad)):
        rel = (got - want).norm() / want.norm()
        assert rel < 2e-2, rel.item()
