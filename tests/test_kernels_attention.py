"""tcgen05 range-masked flash attention vs the fp32 SDPA reference (CQ ranges and varlen samples)."""

import pytest
import torch

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.data.synthetic import synthetic_batch
from cq_pretrain_b200.ops import _ext, attention
from cq_pretrain_b200.ops import reference as R

pytestmark = pytest.mark.gpu


def _check(q, k, v, ks, ke, tol=3e-2):
    args = [t.clone().requires_grad_() for t in (q, k, v)]
    out = attention.cq_attention(*args, ks, ke)
    ref_args = [t.detach().float().requires_grad_() for t in (q, k, v)]
    ref = R.range_attention(*ref_args, ks.cuda(), ke.cuda())
    torch.testing.assert_close(out.float(), ref, atol=tol, rtol=tol)
    g = torch.randn_like(ref)
    out.float().backward(g)
    ref.backward(g)
    for a, b in zip(args, ref_args):
        rel = (a.grad.float() - b.grad).norm() / b.grad.norm().clamp_min(1e-9)
        assert rel < 2e-2, rel.item()


@pytest.mark.parametrize("hd,hq,hkv", [(256, 8, 2), (128, 4, 4), (64, 4, 2)])
def test_cq_ranges(hd, hq, hkv):
    assert _ext.has("attn_fwd")
    cfg = tiny_config(visual_uncond_probability=0.5)
    batch, _ = synthetic_batch(cfg, 512, seed=7, pad_multiple=64)
    plan = batch.mainline
    rows, keys = plan.rows, plan.content_length
    torch.manual_seed(hd)
    q = torch.randn(rows, hq, hd, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(keys, hkv, hd, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(keys, hkv, hd, device="cuda", dtype=torch.bfloat16)
    _check(q, k, v, plan.attn_kstart.cuda(), plan.attn_kend.cuda())


def test_varlen_samples():
    ends = (1024, 1536, 2048)
    ks, ke = attention.ranges_from_ends(ends, ends, "cuda")
    torch.manual_seed(0)
    q = torch.randn(2048, 6, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(2048, 6, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(2048, 6, 128, device="cuda", dtype=torch.bfloat16)
    _check(q, k, v, ks, ke)


def _lse_reference(q, k, ks, ke, scale):
    rep = q.shape[1] // k.shape[1]
    kk = k.float().repeat_interleave(rep, 1)
    s = torch.einsum("rhd,khd->hrk", q.float(), kk) * scale
    keys = torch.arange(k.shape[0], device=q.device)
    allowed = (keys[None] >= ks[:, None].long()) & (keys[None] < ke[:, None].long())
    s = s.masked_fill(~allowed[None], float("-inf"))
    out = torch.logsumexp(s, -1)
    return torch.where(allowed.any(-1)[None], out, torch.full_like(out, float("inf")))


@pytest.mark.parametrize("hd,hq,hkv,amp", [(256, 8, 2, 1.0), (128, 4, 4, 1.0), (64, 4, 2, 1.0), (128, 2, 1, 12.0)])
def test_fwd_lse(hd, hq, hkv, amp):
    """Forward output and LSE (TMEM scores and output, lazy rescale) vs the fp32 reference; amp > 1
    makes the logits large so rows rescale many times."""
    cfg = tiny_config(visual_uncond_probability=0.5)
    batch, _ = synthetic_batch(cfg, 512, seed=5, pad_multiple=64)
    plan = batch.mainline
    ks, ke = plan.attn_kstart.cuda().int(), plan.attn_kend.cuda().int()
    torch.manual_seed(hd + hq)
    q = (torch.randn(plan.rows, hq, hd, device="cuda") * amp).to(torch.bfloat16)
    k = torch.randn(plan.content_length, hkv, hd, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(plan.content_length, hkv, hd, device="cuda", dtype=torch.bfloat16)
    scale = hd ** -0.5
    ops = _ext.ops()
    ops.attn_status(True)
    o, lse = ops.attn_fwd(q, k, v, ks, ke, scale)
    torch.cuda.synchronize()
    assert ops.attn_status() == 0
    ref = R.range_attention(q.float(), k.float(), v.float(), ks, ke, scale)
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)
    want = _lse_reference(q, k, ks, ke, scale)
    finite = torch.isfinite(want)
    assert torch.equal(torch.isfinite(lse), finite)
    torch.testing.assert_close(lse[finite], want[finite], atol=1e-3 * amp, rtol=1e-4)


def test_fwd_varlen_tail():
    """Row count not a multiple of the 128-row block, several samples per block, GQA 3:1."""
    ends = (200, 333, 700, 1000)
    ks, ke = attention.ranges_from_ends(ends, ends, "cuda")
    torch.manual_seed(3)
    q = torch.randn(1000, 6, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1000, 2, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1000, 2, 128, device="cuda", dtype=torch.bfloat16)
    o, _ = _ext.ops().attn_fwd(q, k, v, ks.int(), ke.int(), 128 ** -0.5)
    ref = R.range_attention(q.float(), k.float(), v.float(), ks, ke)
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)
    assert _ext.ops().attn_status() == 0


def _grads_reference(q, k, v, ks, ke, scale, do):
    ref = [t.detach().float().requires_grad_() for t in (q, k, v)]
    R.range_attention(*ref, ks, ke, scale).backward(do.float())
    return [t.grad for t in ref]


def _rel(a, b):
    return ((a.float() - b).norm() / b.norm().clamp_min(1e-9)).item()


@pytest.mark.parametrize("hd,hq,hkv", [(256, 8, 2), (128, 4, 4), (64, 4, 2)])
def test_bwd_cq(hd, hq, hkv):
    """dQ and dK/dV kernels vs fp32 autograd through the reference, CQ ranges."""
    cfg = tiny_config(visual_uncond_probability=0.5)
    batch, _ = synthetic_batch(cfg, 512, seed=13, pad_multiple=64)
    plan = batch.mainline
    ks, ke = plan.attn_kstart.cuda().int(), plan.attn_kend.cuda().int()
    torch.manual_seed(hd * 3 + hq)
    q = torch.randn(plan.rows, hq, hd, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(plan.content_length, hkv, hd, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(plan.content_length, hkv, hd, device="cuda", dtype=torch.bfloat16)
    scale = hd ** -0.5
    ops = _ext.ops()
    ops.attn_status(True)
    o, lse = ops.attn_fwd(q, k, v, ks, ke, scale)
    do = torch.randn_like(o)
    dq, dk, dv = ops.attn_bwd(do, q, k, v, o, lse, ks, ke, scale)
    torch.cuda.synchronize()
    assert ops.attn_status() == 0
    for got, want in zip((dq, dk, dv), _grads_reference(q, k, v, ks, ke, scale, do)):
        assert _rel(got, want) < 2e-2


def test_bwd_varlen_tail():
    """Rows and keys not multiples of the 64/128 tiles, samples straddling blocks, GQA 3:1."""
    ends = (200, 333, 700, 1000)
    ks, ke = attention.ranges_from_ends(ends, ends, "cuda")
    ks, ke = ks.int(), ke.int()
    torch.manual_seed(4)
    q = torch.randn(1000, 6, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1000, 2, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1000, 2, 128, device="cuda", dtype=torch.bfloat16)
    scale = 128 ** -0.5
    ops = _ext.ops()
    o, lse = ops.attn_fwd(q, k, v, ks, ke, scale)
    do = torch.randn_like(o)
    dq, dk, dv = ops.attn_bwd(do, q, k, v, o, lse, ks, ke, scale)
    for got, want in zip((dq, dk, dv), _grads_reference(q, k, v, ks, ke, scale, do)):
        assert _rel(got, want) < 2e-2
    assert ops.attn_status() == 0
