"""CPU tests: CQ planning semantics, chunked gated delta rule and the query-isolation contract."""

import copy

import numpy as np
import torch

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.data.synthetic import synthetic_batch
from cq_pretrain_b200.data.plan import build_plan
from cq_pretrain_b200.ops import reference as R
from cq_pretrain_b200.models.qwen35 import GatedDelta, QwenBlock


def _dense_reference_mask(batch, plan):
    """Reference semantics from sigma/segments (the dense mask the reference would build)."""
    s = batch.ids.shape[1]
    seg = batch.segments[0]
    sig = batch.sigma[0]
    rows = plan.rows
    allowed = torch.zeros(rows, s, dtype=torch.bool)
    same = (seg[:, None] == seg[None]) & (seg[:, None] >= 0)
    allowed[:s] = (sig[None, :] <= sig[:, None]) & same
    qp = plan.query_positions
    for j, p in enumerate(qp.tolist()):
        if plan.query_unconditional[j]:
            continue
        allowed[s + j] = (seg == seg[p]) & (seg[p] >= 0) & (sig < sig[p])
    return allowed


def test_row_ranges_equal_dense_cq_mask():
    cfg = tiny_config(visual_uncond_probability=0.5)
    batch, _ = synthetic_batch(cfg, 512, seed=3)
    plan = batch.mainline
    dense = _dense_reference_mask(batch, plan)
    assert torch.equal(plan.dense_mask(), dense)
    assert torch.equal(plan.attn_valid, dense.any(-1))


def test_chunked_equals_recurrent_with_read_events():
    torch.manual_seed(0)
    E, H, D = 150, 2, 16
    q, k, v = (torch.randn(E, H, D, dtype=torch.float64) for _ in range(3))
    g = -torch.rand(E, H, dtype=torch.float64)
    beta = torch.rand(E, H, dtype=torch.float64)
    reads = torch.rand(E) < 0.4  # read-only events: k = v = 0, beta = g = 0
    k[reads] = 0
    v[reads] = 0
    g[reads] = 0
    beta[reads] = 0
    bounds = (0, 37, 37, 150)
    a = R.recurrent_gated_delta(q, k, v, g, beta, bounds)
    b = R.chunk_gated_delta(q, k, v, g, beta, bounds, chunk=16)
    torch.testing.assert_close(a, b, atol=1e-10, rtol=1e-9)


def test_gdn_layer_queries_never_write_state():
    cfg = tiny_config()
    batch, _ = synthetic_batch(cfg, 256, seed=1)
    plan = batch.mainline
    layer = GatedDelta(cfg).double()
    x = torch.randn(plan.rows, cfg.width, dtype=torch.float64)
    s = plan.content_length
    before = layer(x, plan)
    changed = x.clone()
    changed[s:] += 10 * torch.randn_like(changed[s:])
    after = layer(changed, plan)
    torch.testing.assert_close(before[:s], after[:s], atol=0, rtol=0)


def test_attention_block_future_isolation():
    cfg = tiny_config()
    batch, _ = synthetic_batch(cfg, 256, seed=2)
    plan = batch.mainline
    block = QwenBlock(cfg, 3).double()
    x = torch.randn(plan.rows, cfg.width, dtype=torch.float64)
    rope = (plan.rope_cos.double(), plan.rope_sin.double())
    before = block(x, rope, plan)
    s = plan.content_length
    cut = s // 2
    changed = x.clone()
    changed[cut:] += 5 * torch.randn_like(changed[cut:])
    after = block(changed, rope, plan)
    # content rows before `cut` whose visible range ends before `cut` are unchanged
    keep = (plan.attn_kend[:cut] <= cut).nonzero().flatten()
    torch.testing.assert_close(before[keep], after[keep], atol=0, rtol=0)


def test_packed_documents_equal_independent_documents():
    """A document's content outputs do not depend on other documents in the pack."""
    cfg = tiny_config()
    batch, _ = synthetic_batch(cfg, 256, seed=4)
    plan = batch.mainline
    layer = GatedDelta(cfg).double()
    x = torch.randn(plan.rows, cfg.width, dtype=torch.float64)
    seg = batch.segments[0]
    first = int(seg[0])
    doc = (seg == first).nonzero().flatten()
    before = layer(x, plan)
    other = (seg != first) & (seg >= 0)
    changed = x.clone()
    changed[:plan.content_length][other] += 7
    after = layer(changed, plan)
    torch.testing.assert_close(before[doc], after[doc], atol=0, rtol=0)
