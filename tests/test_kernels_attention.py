"""Range-masked flash attention kernels vs the fp32 SDPA reference (CQ ranges and varlen samples)."""

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
