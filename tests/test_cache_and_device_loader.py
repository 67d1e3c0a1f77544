"""Visual cache identity/checksums/atomic publish and the device loader's acknowledged cursor."""

import pytest
import torch

from cq_pretrain_b200.config import tiny_config
from cq_pretrain_b200.data.cache import VisualCache, canonical_digest, encoder_identity
from cq_pretrain_b200.data.device import DeviceLoader
from cq_pretrain_b200.data.packing import ConsumedLoader, Packer
from cq_pretrain_b200.data.preparer import DevicePreparer
from cq_pretrain_b200.data.synthetic import ListDocuments, tiny_pack_documents


def test_visual_cache_roundtrip_and_integrity(tmp_path):
    (tmp_path / "enc").mkdir()
    (tmp_path / "enc" / "model.safetensors").write_bytes(b"weights")
    (tmp_path / "enc" / "config.json").write_text("{}")
    enc = encoder_identity(str(tmp_path / "enc"))
    cache = VisualCache(tmp_path / "cache", enc, dict(max_pixels=1024))
    ident = cache.identity("sha-of-image", clip=[0, 1])
    assert cache.load(ident) is None
    feats = torch.randn(4, 8)
    path = cache.save(ident, features=feats)
    assert path.name == canonical_digest(ident) + ".pt" and path.parent.name == path.name[:2]
    assert torch.equal(cache.load(ident)["features"], feats)
    assert cache.save(ident, features=torch.zeros(4, 8)) == path       # first writer wins
    assert torch.equal(cache.load(ident)["features"], feats)
    payload = torch.load(path, weights_only=True)
    payload["tensors"]["features"] = feats + 1
    torch.save(payload, path)
    with pytest.raises(ValueError, match="checksum"):
        cache.load(ident)
    other = VisualCache(tmp_path / "cache", enc, dict(max_pixels=2048))
    assert other.path(other.identity("sha-of-image", clip=[0, 1])) != path   # preprocessing is identity


def _loader(cfg, state=None):
    docs = tiny_pack_documents(cfg, 256, seed=1)
    packer = Packer(ListDocuments(docs), cfg, 256, state=state)
    return ConsumedLoader(packer, prefetch=2, state=state)


def test_device_loader_acknowledged_cursor_cpu():
    cfg = tiny_config()
    host = _loader(cfg)
    loader = DeviceLoader(host, DevicePreparer(cfg, "cpu"), prefetch=2)
    first = loader.next()
    start = loader.state_dict()
    batch, receipt = loader.acquire(first)
    assert batch.ids.shape[1] == 256
    assert loader.state_dict() == start            # prefetched but not acknowledged
    loader.acknowledge(receipt)
    resumed_state = loader.state_dict()
    second = loader.next()
    loader.close()
    # a loader resumed from the acknowledged state yields the same next pack
    again = DeviceLoader(_loader(cfg, resumed_state), DevicePreparer(cfg, "cpu"), prefetch=1)
    b2, r2 = again.acquire(again.next())
    assert torch.equal(b2.ids, second.batch.ids) and r2["serial"] == second.receipt["serial"]
    again.close()


@pytest.mark.gpu
def test_device_loader_side_stream_gpu():
    cfg = tiny_config()
    host = _loader(cfg)
    loader = DeviceLoader(host, DevicePreparer(cfg, "cuda"), prefetch=2)
    ref = _loader(cfg)
    for _ in range(3):
        item = loader.next()
        batch, receipt = loader.acquire(item)
        want, _ = ref.next()
        assert batch.ids.is_cuda and torch.equal(batch.ids.cpu(), want.ids)
        loader.acknowledge(receipt)
        ref.acknowledge(receipt)
    assert loader.stats["acquired"] == 3
    loader.close()
    ref.close()


def test_prepare_cache_fills_and_skips(tmp_path):
    import json as _json
    import numpy as np
    from cq_pretrain_b200.data.cache import caches
    from cq_pretrain_b200.data.prepare_cache import prepare
    cfg = tiny_config(vision_min_pixels=32 * 32, vision_max_pixels=64 * 64)
    rng = np.random.default_rng(0)
    rows = []
    for i in range(2):
        pixels = (rng.random((40, 56, 3)) * 255).astype(np.uint8).tolist()
        rows.append(dict(id=f"d{i}", elements=[dict(type="text", input_ids=[5, 6]),
                                                dict(type="image", grid=[1, 2, 4], source=f"sha-{i}", pixels=pixels)]))
    corpus = tmp_path / "corpus"
    corpus.mkdir()
    (corpus / "part.jsonl").write_text("\n".join(_json.dumps(r) for r in rows))
    counts = prepare(cfg, corpus, tmp_path / "cache")
    assert counts["features"] == 2 and counts["latents"] == 2
    again = prepare(cfg, corpus, tmp_path / "cache")
    assert again["features"] == 0 and again["latents"] == 0 and again["skipped"] == 2
    qwen, wan = caches(cfg)
    feats = qwen.load(qwen.identity("sha-0", None))["features"]
    assert feats.shape[1] == cfg.width
    assert wan.load(wan.identity("sha-1", None))["latent"].shape[0] == cfg.latent_channels


def test_stream_attaches_cached_visuals(tmp_path):
    import json as _json
    from cq_pretrain_b200.data.cache import caches
    from cq_pretrain_b200.data.stream import DocumentStream
    cfg = tiny_config()
    cfg.visual_cache = str(tmp_path / "cache")
    qwen, wan = caches(cfg)
    qwen.save(qwen.identity("img-a", None), features=torch.ones(4, cfg.width))
    wan.save(wan.identity("img-a", None), latent=torch.zeros(16, 1, 4, 4))
    corpus = tmp_path / "corpus"
    corpus.mkdir()
    (corpus / "p.jsonl").write_text(_json.dumps(dict(id="d", elements=[
        dict(type="text", input_ids=[7]), dict(type="image", grid=[1, 4, 4], source="img-a")])))
    stream = DocumentStream(corpus, caches=(qwen, wan))
    image = stream.peek()["elements"][1]
    assert torch.equal(image["features"], torch.ones(4, cfg.width)) and image["latent_shape"] == (16, 1, 4, 4)
