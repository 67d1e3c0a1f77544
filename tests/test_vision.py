"""Vision preprocessing (smart resize, patchify in merge order, bilinear positions) and the tower."""

import numpy as np
import torch

from cq_pretrain_b200.data.vision import VisionLayout, patchify, preprocess_image, smart_size
from cq_pretrain_b200.models.vision import VisionTower


def test_smart_size_bounds_and_factor():
    for hw in [(100, 100), (1000, 3000), (4000, 4000), (31, 64)]:
        h, w = smart_size(*hw)
        assert h % 32 == 0 and w % 32 == 0
        assert 65536 * 0.5 <= h * w <= 1048576
    assert smart_size(512, 512) == (512, 512)


def test_patchify_merge_groups_are_contiguous():
    frames = torch.arange(2 * 3 * 64 * 64, dtype=torch.float32).reshape(2, 3, 64, 64)
    patches, grid = patchify(frames)
    assert grid == (1, 4, 4) and patches.shape == (16, 3 * 2 * 16 * 16)
    # row 1 is the (0, 1) patch of the first 2x2 group: pixels at columns 16..31 of row 0
    first = patches[1].reshape(3, 2, 16, 16)
    assert torch.equal(first[0, 0], frames[0, 0, :16, 16:32])
    # row 2 is the (1, 0) patch: rows 16..31, columns 0..15
    assert torch.equal(patches[2].reshape(3, 2, 16, 16)[0, 1], frames[1, 0, 16:32, :16])


def test_preprocess_and_tower_shapes():
    rgb = (np.random.default_rng(0).random((300, 200, 3)) * 255).astype(np.uint8)
    patches, grid = preprocess_image(rgb, min_pixels=64 * 64, max_pixels=128 * 128)
    t, h, w = grid
    assert patches.shape == (t * h * w, 1536)
    assert patches.abs().max() <= 1.0 + 1e-6
    cfg = dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, num_position_embeddings=256,
               out_hidden_size=48)
    tower = VisionTower(cfg, out_width=48, freeze_encoder=False, freeze_merger=False)
    layout = VisionLayout.prepare(patches, [grid], num_positions=256, head_dim=16)
    assert torch.allclose(layout.pos_weights.sum(0), torch.ones(patches.shape[0]))
    assert layout.cos.shape == (patches.shape[0], 16)
    out = tower(layout)
    assert out.shape == (t * (h // 2) * (w // 2), 48)
    out.square().mean().backward()
    assert tower.patch_embed.weight.grad is not None and tower.merger_fc2.weight.grad is not None


def test_frozen_tower_has_no_grad_and_blocks_are_independent():
    torch.manual_seed(0)
    cfg = dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, num_position_embeddings=64,
               out_hidden_size=16)
    tower = VisionTower(cfg)
    a = torch.randn(16, 1536)
    b = torch.randn(16, 1536)
    both = VisionLayout.prepare(torch.cat((a, b)), [(1, 4, 4), (1, 4, 4)], num_positions=64, head_dim=16)
    alone = VisionLayout.prepare(a, [(1, 4, 4)], num_positions=64, head_dim=16)
    out = tower(both)
    assert not out.requires_grad
    assert torch.allclose(out[:4], tower(alone), atol=1e-5)
