"""GDN chunk-recurrence kernels vs the float64 chunked/recurrent oracle (forward and gradients)."""

import pytest
import torch

from cq_pretrain_b200.ops import _ext
from cq_pretrain_b200.ops import reference as R
from cq_pretrain_b200.ops.gdn_cuda import gated_delta_cuda

pytestmark = pytest.mark.gpu


def _inputs(E, H, reads=0.3, seed=0):
    torch.manual_seed(seed)
    q = torch.randn(E, H, 128, device="cuda")
    k = torch.randn(E, H, 128, device="cuda")
    v = torch.randn(E, H, 128, device="cuda")
    g = -torch.rand(E, H, device="cuda") * 0.5
    beta = torch.rand(E, H, device="cuda")
    r = torch.rand(E, device="cuda") < reads
    k[r] = 0
    v[r] = 0
    g[r] = 0
    beta[r] = 0
    return q, k, v, g, beta


@pytest.mark.parametrize("bounds", [(0, 64), (0, 200), (0, 37, 300, 301, 520)])
def test_gdn_forward_backward(bounds):
    assert _ext.has("gdn_fwd")
    E, H = bounds[-1], 4
    q, k, v, g, beta = _inputs(E, H)
    args = [t.clone().requires_grad_() for t in (q, k, v, g, beta)]
    out = gated_delta_cuda(args[0].to(torch.bfloat16), args[1].to(torch.bfloat16), args[2].to(torch.bfloat16),
                           args[3], args[4], bounds)
    ref_args = [t.detach().double().requires_grad_() for t in (q, k, v, g, beta)]
    ref = R.chunk_gated_delta(*ref_args, bounds)
    scale = ref.abs().mean().item()
    err = (out.double() - ref).abs().max().item()
    assert err < 0.08 * max(scale, 1e-3) + 2e-2, (err, scale)
    grad = torch.randn_like(ref)
    out.double().backward(grad)
    ref.backward(grad)
    for name, a, b in zip("qkvgb", args, ref_args):
        rel = (a.grad.double() - b.grad).norm() / b.grad.norm().clamp_min(1e-12)
        assert rel < 5e-2, (name, rel.item())
