"""Cached CQ decoding equals full-prefix recomputation (float64); flow sampler and suite plumbing."""

import numpy as np
import pytest
import torch

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.data.packing import Packer
from cq_pretrain_b200.data.synthetic import ListDocuments
from cq_pretrain_b200.eval import sampling
from cq_pretrain_b200.models.decoding import CQDecoder
from cq_pretrain_b200.models.joint import JointModel


def _one_doc(cfg, ids, length):
    """One templated document whose last body token is the decode placeholder and the only query."""
    doc = dict(id="d", elements=[dict(type="text", input_ids=np.asarray(ids), supervised=False)], templated=False)
    packer = Packer(ListDocuments([doc]), cfg, length)
    batch, _ = packer.next()
    s = len(ids)
    batch.ids, batch.segments = batch.ids[:, :s], batch.segments[:, :s]
    batch.sigma, batch.positions = batch.sigma[:, :s], batch.positions[:, :s]
    batch.image_queries = batch.image_queries[:, :s]
    batch.text_indices = torch.tensor([s - 1])
    from cq_pretrain_b200.data.plan import build_plan
    batch.mainline = build_plan(batch, cfg)
    return batch


def test_cached_decode_matches_full_prefix():
    torch.manual_seed(0)
    cfg = tiny_config(layers=4, vocab_size=128, width=64, ffn=128, heads=4, kv_heads=2, head_dim=16,
                      mrope_section=(1, 1, 0), linear_heads=2, linear_head_dim=16, dit_width=32, dit_heads=2,
                      dit_ffn=64, dit_layers=1, text_mask_token_id=4, image_mask_token_id=5)
    model = JointModel(cfg).double().eval()
    prefix = [10, 11, 12, 13, 14, 15, 3]     # last id is the placeholder of the next token
    decoder = CQDecoder(model, _one_doc(cfg, prefix, 32), max_new_tokens=3)
    full = model.backbone(_one_doc(cfg, prefix, 32))[len(prefix) - 1]
    torch.testing.assert_close(decoder.hidden[0], full, atol=1e-10, rtol=1e-9)
    seq = list(prefix[:-1])
    for token in (21, 22):
        hidden = decoder.advance(token)[0]
        seq.append(token)
        batch = _one_doc(cfg, seq + [3], 32)
        ref = model.backbone(batch)[len(seq)]
        torch.testing.assert_close(hidden, ref, atol=1e-9, rtol=1e-8)


def test_flow_sigmas_and_greedy():
    s = sampling.flow_sigmas(4, 5.0)
    assert s[0] == 1 and s[-1] == 0 and torch.all(s[1:] < s[:-1])
    cfg = tiny_config(layers=4, vocab_size=64, width=32, ffn=64, heads=2, kv_heads=1, head_dim=16,
                      mrope_section=(1, 1, 0), linear_heads=2, linear_head_dim=16, dit_width=32, dit_heads=2,
                      dit_ffn=64, dit_layers=1, text_mask_token_id=4, image_mask_token_id=5)
    model = JointModel(cfg)
    h = torch.randn(1, 32)
    token = sampling.greedy_token(model, h)
    assert token == int((h @ model.embedding.weight.T).argmax())


def test_generate_runs_on_cpu():
    torch.manual_seed(1)
    cfg = tiny_config(layers=4, dit_layers=1)
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    batch, _ = synthetic_batch(cfg, 256, seed=0)
    model = JointModel(cfg).eval()
    out = sampling.generate(model, batch, steps=2, shift=5.0)
    assert out["latent"].shape == (sum(batch.generation.lengths), 64)
    assert torch.isfinite(out["latent"]).all()


@pytest.mark.gpu
def test_graphed_decode_matches_eager_cuda():
    """CUDA-graph replay of the decode step (fixed KV buffers, device-side count and position)
    follows the eager decoder token by token (bf16 model, tcgen05 attention vs SDPA)."""
    from cq_pretrain_b200.models.decoding import GraphedCQDecoder
    torch.manual_seed(0)
    cfg = tiny_config(layers=4, vocab_size=128, width=128, ffn=256, heads=4, kv_heads=2, head_dim=64,
                      mrope_section=(4, 4, 0), linear_heads=2, linear_value_heads=8, linear_head_dim=64, dit_width=32, dit_heads=2,
                      dit_ffn=64, dit_layers=1, text_mask_token_id=4, image_mask_token_id=5)
    model = JointModel(cfg).cuda().to(torch.bfloat16).eval()
    prefix = [10, 11, 12, 13, 14, 15, 3]
    eager = CQDecoder(model, _one_doc(cfg, prefix, 32), max_new_tokens=5)
    graphed = GraphedCQDecoder(model, _one_doc(cfg, prefix, 32), max_new_tokens=5)
    torch.testing.assert_close(graphed.hidden.float(), eager.hidden.float())
    for token in (21, 22, 23, 24):
        want = eager.advance(token).float().clone()
        got = graphed.advance(token).float().clone()
        rel = ((got - want).norm() / want.norm()).item()
        assert rel < 3e-2, (token, rel)
    assert graphed.graph is not None


def test_suite_writes_media_and_reference_scores(tmp_path):
    import json as _json
    from cq_pretrain_b200.data.preparer import DevicePreparer
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    from cq_pretrain_b200.eval.media import latent_preview, reference_scores, save_visual
    from cq_pretrain_b200.parallel import state as ps
    ps.initialize(1)
    cfg = tiny_config()
    model = JointModel(cfg).eval()
    host, receipt = synthetic_batch(cfg, 512, seed=0, pad_multiple=8)
    batch = DevicePreparer(cfg, torch.device("cpu"), torch.float32)(host, receipt)
    scores = reference_scores(model, batch)
    assert scores["text_nll"] > 0 and scores["flow_mse"] > 0 and scores["generation_targets"] == 2
    png = save_visual(np.zeros((8, 8, 3), np.uint8), tmp_path / "still")
    anim = save_visual(np.random.rand(4, 8, 8, 3), tmp_path / "clip", fps=4)
    assert png.suffix == ".png" and png.exists() and anim.suffix in (".mp4", ".webp") and anim.exists()
    preview = latent_preview(torch.randn(16, 2, 6, 6))
    assert preview.shape == (2, 6, 6, 3) and preview.dtype == np.uint8

    def runner(model_, case):
        return dict(score=case["id"], latents=[torch.randn(16, 1, 4, 4)])

    results = sampling.run_suite(model, [dict(id="a", task="t2i"), dict(id="b", task="t2v")], tmp_path / "suite", runner)
    assert [r["media_kind"] for r in results] == ["latent preview"] * 2
    report = (tmp_path / "suite" / "report.html").read_text()
    assert "media/a_0.png" in report and _json.loads((tmp_path / "suite" / "results.json").read_text())[1]["id"] == "b"
