"""MOSS-Image-Base renderer (legacy): four-axis RoPE layout, packing, training step, TP equivalence
over gloo ranks, pointwise CUDA kernels vs the fp32 formulas."""

import os
from pathlib import Path

import numpy as np
import pytest
import torch

from cq_pretrain_b200.config import RunConfig, tiny_config
from cq_pretrain_b200.data.generation import MossGenerationInputs, moss_rope
from cq_pretrain_b200.ops import activation as A

CONFIGS = Path(__file__).resolve().parents[1] / "cq_pretrain_b200" / "configs" / "legacy"


def _cfg(cross=False, fused=True):
    return tiny_config(renderer="moss", latent_channels=8, dit_width=64, dit_heads=4, dit_layers=2, dit_ffn=128,
                       moss_fused_qkv=fused, moss_cross_attention=cross, image_condition_queries=4,
                       visual_query_mode="fixed")


def test_moss_rope_axes():
    cos, sin = moss_rope(2, 3, 4, 16)
    assert cos.shape == (2 * 3 + 4, 16) and sin.shape == cos.shape
    n = 16 // 8
    bands = 1 / (10000.0 ** (torch.arange(n) / n))
    # image token (1, 2): axes (0, text_length, 1 - 0.5, 2 - 1)
    phase = torch.cat([c * bands for c in (0.0, 4.0, 0.5, 1.0)])
    torch.testing.assert_close(cos[5], torch.cat((phase.cos(), phase.cos())))
    torch.testing.assert_close(sin[5], torch.cat((phase.sin(), phase.sin())))
    # condition 3: axes (0, 3, 0, 0)
    phase = torch.cat([c * bands for c in (0.0, 3.0, 0.0, 0.0)])
    torch.testing.assert_close(cos[6 + 3], torch.cat((phase.cos(), phase.cos())))


def test_moss_layout_and_slices():
    layout = MossGenerationInputs.prepare([(4, 6), (2, 2), (3, 3)], [3, 3, 3], 16, token_budget=30)
    assert layout.ends == (27, 34, 46) and layout.text_ends == (3, 6, 9) and layout.video_ends == (24, 28, 37)
    assert layout.video_indices[:3].tolist() == [0, 1, 2] and layout.text_indices[:3].tolist() == [24, 25, 26]
    assert layout.sample_indices.tolist().count(1) == 7
    torch.testing.assert_close(layout.loss_weights.sum(), torch.tensor(1.0))
    parts = layout.microbatches
    assert [(p.start, p.stop) for p in parts] == [(0, 1), (1, 3)]
    second = parts[1].layout
    assert second.ends == (7, 19) and second.video_ends == (4, 13)
    assert second.text_indices.tolist() == [4, 5, 6, 16, 17, 18]
    torch.testing.assert_close(second.cos, layout.cos[27:46])
    with pytest.raises(ValueError):
        MossGenerationInputs.prepare([(8, 8)], [4], 16, token_budget=60)


def test_moss_legacy_configs_load():
    for name in ("qwen35_9b_moss", "qwen35_9b_moss_documents", "qwen35_9b_moss_q64", "qwen35_9b_moss_q64_cross"):
        cfg = RunConfig.load(CONFIGS / f"{name}.json")
        cfg.validate(2)
        assert cfg.renderer == "moss" and cfg.latent_channels == 128 and cfg.dit_layers == 42
    assert RunConfig.load(CONFIGS / "qwen35_9b_moss_q64_cross.json").moss_cross_attention


def _moss_batch(cfg, seed=3, images=2):
    from cq_pretrain_b200.data.synthetic import synthetic_batch
    return synthetic_batch(cfg, 256, seed=seed, kind="joint", images=images, grid=(1, 8, 8),
                           latent_shape=(cfg.latent_channels, 4, 4), understanding=False)


@pytest.mark.parametrize("cross", [False, True])
def test_moss_training_step(cross):
    from cq_pretrain_b200.train.trainer import Trainer
    cfg = _cfg(cross=cross)
    batch, receipt = _moss_batch(cfg)
    assert isinstance(batch.generation, MossGenerationInputs)
    assert batch.latents.shape == (sum(batch.generation.lengths), cfg.latent_channels)
    trainer = Trainer(cfg, tp=1, lr=1e-3, device="cpu", dtype=torch.float32, ema_decay=None, seed=1)
    renderer = trainer.model.renderer
    assert renderer.cross_conditioning == cross
    first = trainer.train_step([(batch, receipt)])
    assert np.isfinite(first["loss"]) and first["image_loss"] > 0
    grads = [p for n, p in renderer.named_parameters() if "text_embedder" in n]
    assert grads and all(p.requires_grad for p in grads)
    second = trainer.train_step([(batch, receipt)])
    assert np.isfinite(second["loss"])


def test_moss_official_names():
    from cq_pretrain_b200.models.moss import MOSSRenderer
    renderer = MOSSRenderer(_cfg(fused=True))
    names = renderer.official_tensors()
    assert "layers.0.proj.q.weight" in names and "layers.0.proj.qkv.weight" not in names
    assert names["layers.0.proj.q.weight"].shape == (64, 64) and "rope.bands" in names
    assert not any(".cross_attn." in n for n in names)
    cross = MOSSRenderer(_cfg(cross=True))
    assert cross.initialize_cross_attention() == 3 * 2


def _moss_inputs(cfg):
    torch.manual_seed(7)
    layout = MossGenerationInputs.prepare([(4, 4), (2, 4)], [4, 4], cfg.dit_width // cfg.dit_heads)
    n = sum(layout.lengths)
    layout.time_features = torch.randn(2, 256)
    batch = type("B", (), {})()
    batch.generation, batch.latents, batch.noise = layout, torch.randn(n, cfg.latent_channels), torch.randn(n, cfg.latent_channels)
    batch.times = torch.tensor([0.3, 0.8])
    conditions = torch.randn(2, 4, cfg.width)
    return conditions, batch


def _moss_tp_worker(rank, world, store, reference):
    import torch.distributed as dist
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    from cq_pretrain_b200.models.moss import MOSSRenderer
    from cq_pretrain_b200.parallel import layers as P
    from cq_pretrain_b200.parallel import state as ps
    ps.initialize(world, backend="gloo", device="cpu")
    saved = torch.load(reference)
    for cross in (False, True):
        cfg = _cfg(cross=cross)
        model = MOSSRenderer(cfg)
        with torch.no_grad():
            for name, p in model.named_parameters():
                p.copy_(P.checkpoint_shard(saved[cross]["state"][name], p))
        conditions, batch = _moss_inputs(cfg)
        conditions.requires_grad_()
        loss = model(conditions, batch)
        torch.testing.assert_close(loss, saved[cross]["loss"], atol=1e-5, rtol=1e-5)
        loss.backward()
        torch.testing.assert_close(conditions.grad, saved[cross]["dcond"], atol=1e-5, rtol=1e-4)
        for name, p in model.named_parameters():
            want = P.checkpoint_shard(saved[cross]["grads"][name], p)
            got = p.grad
            if not getattr(p, "tensor_model_parallel", False) and not getattr(p, "tp_duplicate", False):
                got = got.clone()            # per-head norms: partial over local heads, summed over TP
                dist.all_reduce(got)
                assert name.endswith("q_norm.weight") or name.endswith("k_norm.weight"), name
            torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-4, msg=name)
    dist.destroy_process_group()


def test_moss_tp_matches_single_rank(tmp_path):
    """TP = 2 over gloo: loss, condition gradient and every parameter gradient (sharded ones
    sliced) equal a single-rank run from the same weights, with and without cross-attention."""
    import torch.multiprocessing as mp
    from cq_pretrain_b200.models.moss import MOSSRenderer
    saved = {}
    for cross in (False, True):
        cfg = _cfg(cross=cross)
        torch.manual_seed(2)
        model = MOSSRenderer(cfg)
        with torch.no_grad():   # non-trivial modulation / gates
            for p in model.parameters():
                p.add_(torch.randn_like(p) * 0.05)
        conditions, batch = _moss_inputs(cfg)
        conditions.requires_grad_()
        loss = model(conditions, batch)
        loss.backward()
        saved[cross] = dict(state={n: p.detach().clone() for n, p in model.named_parameters()},
                            grads={n: p.grad.clone() for n, p in model.named_parameters()},
                            loss=loss.detach(), dcond=conditions.grad.clone())
    reference = tmp_path / "reference.pt"
    torch.save(saved, reference)
    mp.spawn(_moss_tp_worker, args=(2, str(tmp_path / "store"), str(reference)), nprocs=2, join=True)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_moss_pointwise_kernels(dtype):
    """situ / affine / gated_add kernels (fwd + bwd, strided column slices) vs fp32 autograd."""
    from cq_pretrain_b200.ops import _ext
    assert _ext.has("moss_pointwise_fwd")
    torch.manual_seed(0)
    fused = (torch.randn(300, 3 * 256, device="cuda") * 6).to(dtype)
    a, b, c = fused[:, :256], fused[:, 256:512], fused[:, 512:]       # strided row slices
    cases = ((A.situ, A.situ_reference, (a, b)), (A.affine, A.affine_reference, (a, b, c)),
             (A.gated_add, A.gated_add_reference, (a, b, c)))
    for fast, slow, args in cases:
        xs = [t.detach().clone().requires_grad_() for t in args]
        ref = [t.detach().float().requires_grad_() for t in args]
        y = fast(*xs)
        want = slow(*ref)
        tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
        torch.testing.assert_close(y.float(), want, atol=tol * want.abs().max().item(), rtol=tol)
        g = torch.randn_like(want)
        y.float().backward(g)
        want.backward(g)
        for got, exp in zip(xs, ref):
            torch.testing.assert_close(got.grad.float(), exp.grad, atol=tol * exp.grad.abs().max().item(), rtol=tol)


def test_moss_codec_pack_and_normalize():
    from cq_pretrain_b200.data import moss_codec as MC
    x = torch.arange(2 * 3 * 4 * 6, dtype=torch.float32).reshape(2, 3, 4, 6)
    p = MC.pack(x)
    assert p.shape == (2, 12, 2, 3)
    # channel (c=1, dy=1, dx=0) of token (1, 2) is pixel (2*1+1, 2*2+0) of channel 1
    assert p[0, 1 * 4 + 2, 1, 2] == x[0, 1, 3, 4]
    mean, std = torch.randn(1, 3, 4, 6), torch.rand(1, 3, 4, 6)
    rm, rv = torch.randn(12), torch.rand(12) + 0.5
    m, s = MC.normalize_posterior(mean, std, rm, rv, 1e-4)
    torch.testing.assert_close(m, (MC.pack(mean) - rm.view(1, -1, 1, 1)) / (rv.view(1, -1, 1, 1) + 1e-4).sqrt())
    torch.testing.assert_close(s, MC.pack(std) / (rv.view(1, -1, 1, 1) + 1e-4).sqrt())
    z = MC.draw_latents([m[0]], [s[0]], torch.Generator().manual_seed(0))
    assert z.shape == (6, 12)
