"""LM-head cross-entropy with the GEMM statistics / gradient epilogues vs fp32 PyTorch."""

import pytest
import torch

from cq_pretrain_b200.ops import _ext
from cq_pretrain_b200.ops.cross_entropy import linear_cross_entropy

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,vocab,chunk", [(300, 4096, 128), (1024, 248320 // 8, 1024), (77, 1000, 64)])
def test_linear_ce_matches_fp32(rows, vocab, chunk):
    assert _ext.has("ce_stats") and _ext.has("ce_grad_logits")
    torch.manual_seed(0)
    h = (torch.randn(rows, 256, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    w = (torch.randn(vocab, 256, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_()
    t = torch.randint(0, vocab, (rows,), device="cuda")
    loss = linear_cross_entropy(h, w, t, chunk)
    loss.backward()
    hr, wr = h.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    ref = torch.nn.functional.cross_entropy(hr @ wr.T, t)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 2e-3 * max(1.0, abs(ref.item()))
    for got, want in ((h.grad, hr.grad), (w.grad, wr.grad)):
        rel = (got.float() - want).norm() / want.norm()
        assert rel < 2e-2, rel.item()


def test_ce_stats_partial_shard():
    torch.manual_seed(1)
    h = torch.randn(130, 128, device="cuda").to(torch.bfloat16)
    w = torch.randn(592, 128, device="cuda").to(torch.bfloat16)
    t = torch.randint(0, 1200, (130,), device="cuda")
    mx, tgt, se = _ext.ops().ce_stats(h, w, t, 600)   # this shard holds ids [600, 1192)
    logits = (h.float() @ w.float().T)
    torch.testing.assert_close(mx, logits.max(-1).values, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(se, torch.exp(logits - mx[:, None]).sum(-1), rtol=2e-3, atol=1e-3)
    owned = (t >= 600) & (t < 1192)
    want = torch.where(owned, logits.gather(1, (t - 600).clamp(0, 591)[:, None])[:, 0], torch.zeros_like(mx))
    torch.testing.assert_close(tgt, want, rtol=1e-3, atol=1e-3)
