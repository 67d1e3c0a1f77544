"""Checkpoint identity pins and the TAR-range image reader (CPU)."""

import hashlib
import io
import json
import tarfile

import numpy as np
import pytest

from cq_pretrain_b200.data.images import ImageReader
from cq_pretrain_b200.utils.assets import asset_manifest, vision_config


def test_asset_manifest_and_vision_guard(tmp_path):
    (tmp_path / "a.bin").write_bytes(b"abc")
    manifest = dict(model_id="Qwen/Qwen3.5-0.8B", revision="2fc06364715b967f1860aea9cf38778875588b17",
                    files={"a.bin": hashlib.sha256(b"abc").hexdigest()})
    (tmp_path / "manifest.json").write_text(json.dumps(manifest))
    assert asset_manifest(tmp_path, verify=True)["model_id"] == "Qwen/Qwen3.5-0.8B"
    (tmp_path / "a.bin").write_bytes(b"abd")
    with pytest.raises(ValueError, match="changed"):
        asset_manifest(tmp_path, verify=True)
    (tmp_path / "manifest.json").write_text(json.dumps(dict(manifest, revision="0" * 40)))
    with pytest.raises(ValueError, match="not pinned"):
        asset_manifest(tmp_path)
    good = dict(patch_size=16, temporal_patch_size=2, spatial_merge_size=2, hidden_act="gelu_pytorch_tanh")
    (tmp_path / "config.json").write_text(json.dumps(dict(vision_config=good)))
    assert vision_config(tmp_path)["patch_size"] == 16
    (tmp_path / "config.json").write_text(json.dumps(dict(vision_config=dict(good, deepstack_visual_indexes=[1]))))
    with pytest.raises(ValueError, match="DeepStack"):
        vision_config(tmp_path)


def test_image_reader_ranges_integrity_and_exif(tmp_path):
    from PIL import Image
    img = Image.fromarray((np.arange(20 * 30 * 3) % 255).astype(np.uint8).reshape(20, 30, 3))
    exif = Image.Exif()
    exif[0x0112] = 6                      # rotate 90 degrees on display
    buf = io.BytesIO()
    img.save(buf, format="JPEG", exif=exif.tobytes())
    payload = buf.getvalue()
    shard = tmp_path / "shard.tar"
    with tarfile.open(shard, "w") as tar:
        info = tarfile.TarInfo("x.jpg")
        info.size = len(payload)
        tar.addfile(info, io.BytesIO(payload))
    with tarfile.open(shard) as tar:
        member = tar.getmember("x.jpg")
    locator = dict(shard="shard.tar", offset=member.offset_data, length=member.size,
                   sha256=hashlib.sha256(payload).hexdigest())
    reader = ImageReader(tmp_path, {"shard.tar": shard.stat().st_size}, native_resolution=True)
    pixels = reader.read(locator)
    assert pixels.shape == (30, 20, 3)      # EXIF orientation applied
    fitted = ImageReader(tmp_path, {"shard.tar": shard.stat().st_size}, image_size=16).read(locator)
    assert fitted.shape == (16, 16, 3)
    with pytest.raises(RuntimeError, match="integrity"):
        reader.read_bytes(dict(locator, sha256="0" * 64))
    with pytest.raises(ValueError):
        reader.read_bytes(dict(locator, shard="../shard.tar"))
    with pytest.raises(ValueError):
        reader.read_bytes(dict(locator, offset=shard.stat().st_size))
    reader.close()


def test_asset_preparer_pins_verifies_and_checks_upstream(tmp_path):
    import hashlib
    import json
    from cq_pretrain_b200.utils import prepare_assets as PA
    src = tmp_path / "src"
    src.mkdir()
    (src / "config.json").write_text(json.dumps(dict(vision_config=dict(patch_size=16, temporal_patch_size=2,
                                                                        spatial_merge_size=2,
                                                                        hidden_act="gelu_pytorch_tanh"))))
    (src / "tokenizer.json").write_text("{}")
    (src / "model.safetensors.index.json").write_text(json.dumps(dict(weight_map={"a": "m-1.safetensors",
                                                                                  "b": "m-2.safetensors"})))
    for n in ("m-1.safetensors", "m-2.safetensors"):
        (src / n).write_bytes(n.encode() * 10)
    model_id, rev = "Qwen/Qwen3.5-2B-Base", "b1485b2fa6dfa1287294f269f5fb618e03d52d7c"
    lfs = {n: hashlib.sha256((src / n).read_bytes()).hexdigest() for n in ("m-1.safetensors", "m-2.safetensors")}
    blob = hashlib.sha1(b"blob 2\0{}").hexdigest()
    meta = dict(sha=rev, siblings=[dict(rfilename=n, lfs=dict(sha256=h)) for n, h in lfs.items()]
                + [dict(rfilename="tokenizer.json", blobId=blob)])
    (tmp_path / "meta.json").write_text(json.dumps(meta))
    out = PA.pin(src, tmp_path / "pinned", model_id, rev, upstream=tmp_path / "meta.json", vision=True)
    assert out["upstream_checked"] and set(out["files"]) >= {"config.json", "m-1.safetensors", "m-2.safetensors"}
    assert PA.verify(tmp_path / "pinned", vision=True)["revision"] == rev
    (tmp_path / "pinned" / "m-2.safetensors").write_bytes(b"tampered")
    with pytest.raises(ValueError, match="changed"):
        PA.verify(tmp_path / "pinned")
    with pytest.raises(ValueError, match="not a pinned"):
        PA.pin(src, tmp_path / "other", model_id, "0" * 40)
    meta["siblings"][0]["lfs"]["sha256"] = "0" * 64
    (tmp_path / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(ValueError, match="upstream"):
        PA.pin(src, tmp_path / "third", model_id, rev, upstream=tmp_path / "meta.json")
