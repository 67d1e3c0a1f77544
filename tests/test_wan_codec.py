"""Wan2.1 VAE codec: geometry, causality of the chunked encode / decode, checkpoint round trip."""

import pytest
import torch

from cq_pretrain_b200.data.wan_codec import LATENT_MEAN, WanVideoCodec
from cq_pretrain_b200.models.wan_vae import WanVAE


def test_published_geometry_and_names():
    with torch.device("meta"):
        vae = WanVAE()
    assert abs(sum(p.numel() for p in vae.parameters()) / 1e6 - 126.9) < 0.1
    keys = vae.state_dict().keys()
    for name in ("encoder.conv1.weight", "encoder.downsamples.0.residual.0.gamma", "encoder.middle.1.to_qkv.weight",
                 "encoder.head.2.weight", "conv1.weight", "conv2.weight", "decoder.upsamples.3.time_conv.weight",
                 "decoder.head.0.gamma"):
        assert name in keys, name


def test_chunked_encode_decode_is_causal_and_shaped():
    torch.manual_seed(0)
    codec = WanVideoCodec(WanVAE(dim=16))
    video = torch.rand(3, 9, 32, 48) * 2 - 1
    z = codec.encode(video)
    assert z.shape == (16, 3, 4, 6)
    # a prefix of the video (an image, or the first 1 + 4 frames) encodes to the same latents
    assert torch.equal(codec.encode(video[:, :1]), z[:, :1])
    assert torch.equal(codec.encode(video[:, :5]), z[:, :2])
    out = codec.decode([z])[0]
    assert out.shape == (3, 9, 32, 48) and out.abs().max() <= 1
    assert torch.equal(codec.decode([z[:, :2]])[0], out[:, :5])
    assert codec.encode_images(video[:, 0][None].repeat(2, 1, 1, 1)).shape == (2, 16, 4, 6)
    frames = codec.frames(z)
    assert frames.shape == (9, 32, 48, 3) and 0 <= frames.min() and frames.max() <= 1
    with pytest.raises(ValueError):
        codec.encode(video[:, :4])


def test_checkpoint_round_trip_and_normalisation(tmp_path):
    torch.manual_seed(1)
    vae = WanVAE(dim=16)
    torch.save(vae.state_dict(), tmp_path / "Wan2.1_VAE.pth")
    loaded = WanVideoCodec.from_pretrained(tmp_path)
    video = torch.rand(3, 5, 16, 16) * 2 - 1
    raw = vae.eval().encode(video[None])[0]
    z = loaded.encode(video)
    mean = torch.tensor(LATENT_MEAN).view(-1, 1, 1, 1)
    assert torch.allclose(z * loaded.std + mean, raw, atol=1e-5)
