"""Sentinel / two-source row gathers (csrc/gather.cu) and their inverse-level backward."""

import numpy as np
import pytest
import torch

from cq_pretrain_b200.ops import _ext
from cq_pretrain_b200.ops import gather as GA

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, (16, 128)), (torch.float32, (8,))])
def test_rows_two_sources_and_sentinel(dtype, shape):
    assert _ext.has("gather_rows")
    rng = np.random.default_rng(0)
    n0, n1, m = 300, 40, 900
    index = rng.integers(0, n0 + n1 + 1, size=m)         # n0 + n1 = sentinel (zeros)
    index[:5] = n0 + n1
    inverse = GA.inverse_levels(index, n0 + n1 + 1, ignore=n0 + n1)
    a = torch.randn(n0, *shape, device="cuda").to(dtype).requires_grad_()
    b = torch.randn(n1, *shape, device="cuda").to(dtype).requires_grad_()
    idx = torch.from_numpy(index).cuda()
    inv = tuple(t.cuda() for t in inverse)
    out = GA.rows(a, idx, inv, second=b)
    ref_src = torch.cat((a.detach().float(), b.detach().float(), torch.zeros(1, *shape, device="cuda")))
    torch.testing.assert_close(out.float(), ref_src[idx])
    g = torch.randn_like(out)
    out.backward(g)
    want = torch.zeros(n0 + n1 + 1, *shape, device="cuda").index_add_(0, idx, g.float())
    torch.testing.assert_close(a.grad.float(), want[:n0], atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(b.grad.float(), want[n0:n0 + n1], atol=2e-2, rtol=1e-2)


def test_rows_strided_source():
    proj = torch.randn(500, 96, device="cuda").to(torch.bfloat16)
    src = proj[:, 16:48].detach().requires_grad_(False)          # column slice: row stride 96
    view = proj[:, 16:48]
    idx = torch.randint(0, 501, (700,), device="cuda")
    out = GA.rows(view, idx)
    ref = torch.cat((src.float(), torch.zeros(1, 32, device="cuda")))[idx]
    torch.testing.assert_close(out.float(), ref)
