"""Fill the immutable visual caches: Qwen merger features and Wan latents of every corpus image.

``python -m cq_pretrain_b200.data.prepare_cache --corpus DIR --cache DIR [--rank r --world w]``
walks this rank's share of the catalog (same sharding as training), and for every image element
that carries pixels (``pixels`` uint8 ``[H, W, 3]`` or a ``path``) and a ``source`` identity
(e.g. the image sha256) computes what is missing:

* merger features: native-resolution preprocessing (``data/vision.py``) → frozen vision tower;
* latents: pixels resized to the generation geometry → the latent encoder (the Wan VAE, ``--latent-encoder wan``, when its
  weights are available; ``FakeLatentEncoder`` for pipeline runs without them).

Entries are content-addressed and published atomically, so any number of ranks can run at once
and a restarted run only computes what is missing (reference ``scripts/prepare_latents.py:14-62``).
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .cache import caches
from .preparer import FakeLatentEncoder
from .stream import DocumentStream
from .vision import VisionLayout, preprocess_image


def _pixels(element):
    if "pixels" in element:
        return np.asarray(element["pixels"], dtype=np.uint8)
    from PIL import Image, ImageOps
    with Image.open(element["path"]) as im:
        return np.asarray(ImageOps.exif_transpose(im).convert("RGB"))


@torch.no_grad()
def prepare(cfg, corpus, cache_root, rank=0, world=1, device="cpu", vision=None, encoder=None, dtype=torch.float32):
    """Returns counts of written/skipped entries. ``vision``: a frozen VisionTower (built if None)."""
    cfg.visual_cache = str(cache_root)
    feature_cache, latent_cache = caches(cfg)
    if vision is None:
        from ..models.vision import VisionTower, vision_config
        vision = VisionTower(vision_config(cfg), cfg.width).to(device=device, dtype=dtype).eval()
    encoder = encoder or FakeLatentEncoder(cfg.latent_channels)
    stream = DocumentStream(corpus, rank=rank, world=world)
    counts = dict(features=0, latents=0, skipped=0, documents=0)
    head_dim = vision.head_dim()
    while (doc := stream.peek()) is not None:
        stream.advance()
        counts["documents"] += 1
        for element in doc["elements"]:
            if element.get("type") != "image" or "source" not in element:
                continue
            if "pixels" not in element and "path" not in element:
                continue
            rgb = None
            fkey = feature_cache.identity(element["source"], element.get("clip"))
            if feature_cache.load(fkey) is None:
                rgb = _pixels(element)
                patches, grid = preprocess_image(rgb, cfg.vision_min_pixels, cfg.vision_max_pixels)
                layout = VisionLayout.prepare(patches.to(device=device, dtype=dtype), [grid],
                                              num_positions=vision.cfg["num_position_embeddings"], head_dim=head_dim)
                layout = layout.to(device)
                feature_cache.save(fkey, features=vision(layout).float().cpu(), grid=torch.tensor(grid))
                counts["features"] += 1
            else:
                counts["skipped"] += 1
            lkey = latent_cache.identity(element["source"], element.get("clip"))
            if latent_cache.load(lkey) is None:
                rgb = _pixels(element) if rgb is None else rgb
                x = torch.from_numpy(rgb).permute(2, 0, 1)[None].float().div(127.5).sub(1)
                h = max(16, (x.shape[2] // 16) * 16)
                w = max(16, (x.shape[3] // 16) * 16)
                x = torch.nn.functional.interpolate(x, size=(h, w), mode="bilinear", align_corners=False)
                images = getattr(encoder, "encode_images", None)     # the Wan codec: one-frame videos
                latent = images(x.to(device)) if images is not None else encoder.encode(x.to(device))
                if isinstance(latent, tuple):    # posterior (mean, std) encoders cache the mean
                    latent = latent[0]
                latent = latent[:, :, None]      # [1, C, T=1, h/stride, w/stride]
                latent_cache.save(lkey, latent=latent[0].float().cpu())
                counts["latents"] += 1
    stream.close()
    return counts


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--config", default=None, help="YAML run config (default: Qwen3.5-2B + Wan)")
    parser.add_argument("--corpus", required=True)
    parser.add_argument("--cache", required=True)
    parser.add_argument("--rank", type=int, default=0)
    parser.add_argument("--world", type=int, default=1)
    parser.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    parser.add_argument("--latent-encoder", choices=("fake", "kl16", "wan"), default="fake",
                        help="kl16: the legacy renderer's KL16 VAE (needs --kl16-checkpoint); wan: the Wan2.1 VAE "
                             "(needs --wan-vae)")
    parser.add_argument("--kl16-checkpoint", default=None)
    parser.add_argument("--wan-vae", default=None, help="Wan2.1_VAE.pth or the directory holding it")
    args = parser.parse_args(argv)
    from ..config import load_sections, qwen35_2b_wan
    cfg = load_sections(args.config)[0] if args.config else qwen35_2b_wan()
    dtype = torch.bfloat16 if args.device.startswith("cuda") else torch.float32
    encoder = None
    if args.latent_encoder == "kl16":
        if not args.kl16_checkpoint:
            raise SystemExit("--latent-encoder kl16 needs --kl16-checkpoint")
        from ..models.kl16 import FrozenKL16
        encoder = FrozenKL16(args.kl16_checkpoint, dtype=torch.float32, device=args.device)
    elif args.latent_encoder == "wan":
        if not args.wan_vae:
            raise SystemExit("--latent-encoder wan needs --wan-vae")
        from .wan_codec import WanVideoCodec
        encoder = WanVideoCodec.from_pretrained(args.wan_vae, device=args.device)
    counts = prepare(cfg, args.corpus, args.cache, args.rank, args.world, args.device, encoder=encoder, dtype=dtype)
    print(json.dumps(dict(status="complete", **counts)), flush=True)


if __name__ == "__main__":
    main()
