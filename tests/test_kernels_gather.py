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


def test_embedding_lookup_and_sparse_main_grad_backward():
    """Vocabulary embedding on CUDA: row-gather lookup with the zero sentinel for other shards' ids,
    and the deterministic per-id accumulation into main_grad, vs F.embedding + a dense gradient."""
    from cq_pretrain_b200.parallel import layers as PL
    from cq_pretrain_b200.parallel import state as ps
    ps.initialize(1)
    torch.manual_seed(0)
    emb = PL.VocabEmbedding(5000, 256).cuda().to(torch.bfloat16)
    ids = torch.randint(0, 5000, (3000,), device="cuda")
    ids[:500] = 7                                        # a heavily repeated id
    grad = torch.randn(3000, 256, device="cuda").to(torch.bfloat16)
    ref_w = emb.weight.detach().float().requires_grad_()
    ref = torch.nn.functional.embedding(ids, ref_w)
    ref.backward(grad.float())
    out = emb.partial(ids)
    torch.testing.assert_close(out.float(), ref.detach())
    out.backward(grad)                                   # no main_grad: a dense gradient comes back
    torch.testing.assert_close(emb.weight.grad.float(), ref_w.grad, rtol=2e-2, atol=2e-2)
    emb.weight.grad = None
    emb.weight.main_grad = torch.full((5000, 256), 0.5, device="cuda")
    emb.partial(ids).backward(grad)                      # with main_grad: accumulated in place
    assert emb.weight.grad is None
    torch.testing.assert_close(emb.weight.main_grad - 0.5, ref_w.grad, rtol=1e-4, atol=1e-3)
    first = emb.weight.main_grad.clone()
    emb.weight.main_grad.fill_(0.5)
    emb.partial(ids).backward(grad)
    assert torch.equal(first, emb.weight.main_grad)      # deterministic


def test_embedding_backward_with_host_plan_matches_device_sort():
    """The host-built sort plan (``EmbeddingPlan``) gives the same main_grad as the on-device sort,
    including a shard offset (ids of other shards are skipped)."""
    from cq_pretrain_b200.data.batch import EmbeddingPlan
    from cq_pretrain_b200.parallel import layers as PL
    from cq_pretrain_b200.parallel import state as ps
    ps.initialize(1)
    torch.manual_seed(1)
    emb = PL.VocabEmbedding(4000, 128).cuda().to(torch.bfloat16)
    ids = torch.randint(0, 6000, (2500,))                # ids >= 4000 behave like another shard's
    ids[:300] = 11
    plan = EmbeddingPlan.build(ids.numpy()).to("cuda")
    grad = torch.randn(2500, 128, device="cuda").to(torch.bfloat16)
    outs = []
    for p in (None, plan):
        emb.weight.main_grad = torch.zeros(4000, 128, device="cuda")
        emb.partial(ids.cuda(), p).backward(grad)
        outs.append(emb.weight.main_grad.clone())
    assert torch.equal(outs[0], outs[1])
