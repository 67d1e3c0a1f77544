"""tcgen05 GEMM kernels vs fp32 PyTorch references (all three operand layouts, tails included)."""

import pytest
import torch

from cq_pretrain_b200.ops import _ext

pytestmark = pytest.mark.gpu


def _status_ok():
    assert _ext.ops().gemm_status(True) == 0, "GEMM reported a bounded-wait timeout"


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 272, 96), (1000, 512, 2048), (4096, 3072, 1024)])
def test_gemm_nt(m, n, k):
    torch.manual_seed(m + n + k)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    y = _ext.ops().gemm_nt(x, w, b)
    torch.cuda.synchronize()
    _status_ok()
    ref = x.float() @ w.float().T + b.float()
    torch.testing.assert_close(y.float(), ref, atol=3e-2 * (k ** 0.5) * 0.05 + 2e-2, rtol=2e-2)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 320, 80), (2048, 2048, 6144)])
def test_gemm_nn(m, n, k):
    torch.manual_seed(m + 2 * n + k)
    a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(k, n, device="cuda", dtype=torch.bfloat16) * 0.05
    y = _ext.ops().gemm_nn(a, b)
    torch.cuda.synchronize()
    _status_ok()
    ref = a.float() @ b.float()
    torch.testing.assert_close(y.float(), ref, atol=5e-2, rtol=2e-2)


@pytest.mark.parametrize("m,n,k", [(64, 128, 256), (333, 272, 144), (4096, 1024, 2048)])
def test_gemm_tn_accumulate(m, n, k):
    torch.manual_seed(3 * m + n + k)
    a = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    out = torch.randn(n, k, device="cuda", dtype=torch.float32)
    ref = out + a.float().T @ b.float()
    _ext.ops().gemm_tn_acc(a, b, out)
    torch.cuda.synchronize()
    _status_ok()
    torch.testing.assert_close(out, ref, atol=1e-2 * (m ** 0.5), rtol=1e-3)


def test_linear_autograd_uses_kernel():
    from cq_pretrain_b200.ops import linear as L
    torch.manual_seed(0)
    x = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(768, 1024, device="cuda") * 0.02).to(torch.bfloat16).requires_grad_()
    w.main_grad = torch.zeros(768, 1024, device="cuda")
    before = _ext.launches()
    y = L.linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    dx = x.grad
    assert _ext.launches() - before >= 3
    torch.testing.assert_close(y.float(), x.float() @ w.float().T, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(dx.float(), g.float() @ w.float(), atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(w.main_grad, g.float().T @ x.float(), atol=0.5, rtol=1e-2)


@pytest.mark.parametrize("mn_major", [False, True])
def test_dual_operand_pair_gemm(mn_major):
    """Two operand pairs in one k loop (x w + x2 w2, x2 over fewer rows): the pair the GEMM ->
    reduce-scatter kernel runs for two projections of one input, here on one GPU vs fp32."""
    assert _ext.has("gemm_dual")
    torch.manual_seed(2)
    M, N, K, K2, M2 = 640, 384, 256, 160, 440
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    x2 = torch.randn(M2, K2, device="cuda").to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda") * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(K2, N, device="cuda") * 0.05).to(torch.bfloat16)
    if not mn_major:
        w, w2 = w.t().contiguous(), w2.t().contiguous()
    y = _ext.ops().gemm_dual(x, w, x2, w2, mn_major)
    wf, w2f = (w.float(), w2.float()) if mn_major else (w.float().t(), w2.float().t())
    ref = x.float() @ wf
    ref[:M2] += x2.float() @ w2f
    rel = (y.float() - ref).abs().max() / ref.abs().max()
    assert rel < 1e-2, rel.item()
