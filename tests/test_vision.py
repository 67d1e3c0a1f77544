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


def _vision_tp_worker(rank, world, store):
    import os

    import torch.distributed as dist

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    from cq_pretrain_b200.parallel import layers as P
    from cq_pretrain_b200.parallel import state as ps
    ps.initialize(world, backend="gloo", device="cpu")
    cfg = dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, num_position_embeddings=64,
               out_hidden_size=32)
    torch.manual_seed(0)
    full = VisionTower(cfg, freeze_encoder=False, freeze_merger=False)
    sharded = VisionTower(dict(cfg, tensor_parallel=True), freeze_encoder=False, freeze_merger=False)
    pairs = list(zip(sharded.named_parameters(), full.named_parameters()))
    with torch.no_grad():
        for (name, p), (name_full, q) in pairs:
            assert name == name_full
            p.copy_(P.checkpoint_shard(q, p))
    assert sharded.blocks[0].qkv.weight.shape == (96, 64)          # column shard (stride 3)
    assert sharded.blocks[0].proj.weight.shape == (64, 32)         # row shard
    assert sharded.blocks[0].norm1.weight.tp_duplicate
    torch.manual_seed(1)
    layout = VisionLayout.prepare(torch.randn(32, 1536), [(1, 4, 4), (1, 4, 4)], num_positions=64, head_dim=16)
    out_full, out_tp = full(layout), sharded(layout)
    torch.testing.assert_close(out_tp, out_full, atol=1e-5, rtol=1e-5)
    out_full.square().sum().backward()
    out_tp.square().sum().backward()
    for (name, p), (_, q) in pairs:
        torch.testing.assert_close(p.grad, P.checkpoint_shard(q.grad, p), atol=1e-5, rtol=1e-4, msg=name)
    dist.destroy_process_group()


def test_vision_tp_matches_replicated(tmp_path):
    """Vision TP (column qkv/fc1/merger fc1, row proj/fc2/merger fc2) on 2 gloo ranks: outputs
    equal the replicated tower, sharded gradients equal slices of the full ones and replicated
    (tp_duplicate) gradients equal the full ones on every rank."""
    import torch.multiprocessing as mp
    mp.spawn(_vision_tp_worker, args=(2, str(tmp_path / "store")), nprocs=2, join=True)
