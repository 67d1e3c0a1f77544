"""Legacy flow renderer + RGB patch embedding (smoke config, CPU fp32): a full training step."""

from pathlib import Path

import numpy as np
import torch

from cq_pretrain_b200.config import RunConfig
from cq_pretrain_b200.data.packing import Packer
from cq_pretrain_b200.data.synthetic import ListDocuments, text_ids

CONFIGS = Path(__file__).resolve().parents[1] / "cq_pretrain_b200" / "configs" / "legacy"


def _docs(cfg, n_docs=6, seed=0):
    rng = np.random.default_rng(seed)
    side = int(np.sqrt(cfg.image_tokens))
    docs = []
    for i in range(2):
        image = dict(type="image", grid=(1, 2 * side, 2 * side), generation_target=True,
                     pixels=torch.from_numpy(rng.uniform(-1, 1, (3, cfg.image_size, cfg.image_size)).astype(np.float32)),
                     latent_shape=(cfg.latent_channels, 1, side, side),
                     latent=torch.from_numpy(rng.standard_normal((cfg.latent_channels, 1, side, side)).astype(np.float32)))
        docs.append(dict(id=f"v{i}", direction="T2I", format="caption",
                         elements=[dict(type="text", input_ids=text_ids(rng, 12, 1000)), image]))
    for k in range(n_docs):
        docs.append(dict(id=f"t{k}", elements=[dict(type="text", input_ids=text_ids(rng, 40, 1000))]))
    return docs


def test_legacy_configs_load():
    for name in ("qwen35_cq", "qwen35_cq_smoke"):
        cfg = RunConfig.load(CONFIGS / f"{name}.json")
        cfg.validate(1)
        assert cfg.renderer == "legacy"


def test_legacy_renderer_training_step():
    from cq_pretrain_b200.train.trainer import Trainer
    cfg = RunConfig.load(CONFIGS / "qwen35_cq_smoke.json")
    cfg.vocab_size = 2048
    cfg.text_mask_token_id, cfg.image_mask_token_id = 2001, 2002
    packer = Packer(ListDocuments(_docs(cfg)), cfg, 192)
    batch, receipt = packer.next()
    assert batch.latents.shape == (2, cfg.image_tokens, cfg.latent_channels)
    assert batch.vision.pixel_values.shape == (2, 3, cfg.image_size, cfg.image_size)
    trainer = Trainer(cfg, tp=1, lr=1e-3, device="cpu", dtype=torch.float32, ema_decay=None)
    first = trainer.train_step([(batch, receipt)])
    assert np.isfinite(first["loss"]) and first["image_loss"] > 0
    renderer = trainer.model.renderer
    assert renderer.output.weight.abs().sum() > 0          # zero-initialised output layer was trained
    second = trainer.train_step([(batch, receipt)])
    assert np.isfinite(second["loss"])


def test_kl16_encoder_geometry_and_names():
    """KL16 encoder: 16x downsampling to 2 x 16 moments, attention only at the 16x16 level,
    checkpoint parameter names, clamped scaled posterior."""
    from cq_pretrain_b200.models.kl16 import FrozenKL16
    torch.manual_seed(0)
    codec = FrozenKL16(chunk=1)
    names = dict(codec.named_parameters())
    for key in ("encoder.conv_in.weight", "encoder.down.0.block.0.norm1.weight", "encoder.down.2.block.0.nin_shortcut.weight",
                "encoder.down.4.attn.1.proj_out.weight", "encoder.down.3.downsample.conv.weight",
                "encoder.mid.attn_1.q.weight", "encoder.norm_out.weight", "quant_conv.weight"):
        assert key in names, key
    assert not any(k.startswith("encoder.down.3.attn") for k in names)
    assert not any(k.startswith("encoder.down.4.downsample") for k in names)
    pixels = torch.rand(2, 3, 64, 96) * 2 - 1
    mean, std = codec.encode(pixels)
    assert mean.shape == std.shape == (2, 16, 4, 6)
    assert (std > 0).all() and torch.isfinite(mean).all()
    # chunking does not change the result
    one = FrozenKL16(chunk=2)
    one.load_state_dict(codec.state_dict())
    torch.testing.assert_close(one.encode(pixels)[0], mean, atol=1e-5, rtol=1e-5)
