"""Video decoding (NPY), fixed and native clip preparation, tower frame sampling (CPU)."""

import numpy as np
import pytest
import torch

from cq_pretrain_b200.data.video import (decode_video, prepare_fixed_clip, prepare_native_clip, qwen_frame_indices,
                                         qwen_video_patches, wan_latent_shape)


def _npy(tmp_path, t=23, h=48, w=64):
    frames = (np.arange(t * h * w * 3) % 251).astype(np.uint8).reshape(t, h, w, 3)
    frames[:, :, :, 0] = np.arange(t)[:, None, None]      # frame number in the red channel
    path = tmp_path / "clip.npy"
    np.save(path, frames)
    return dict(frames_path=str(path), fps=10.0), frames


def test_decode_and_fixed_clip(tmp_path):
    entry, frames = _npy(tmp_path)
    decoded, times, digest = decode_video(entry)
    assert decoded.shape == frames.shape and np.allclose(np.diff(times), 0.1) and len(digest) == 64
    rgb, clip = prepare_fixed_clip(dict(entry, start_seconds=0.5), num_frames=9, fps=5.0, height=32, width=32)
    assert rgb.shape == (9, 3, 32, 32) and rgb.dtype == torch.uint8
    assert clip["frame_indices"] == [5, 7, 9, 11, 13, 15, 17, 19, 21]
    with pytest.raises(ValueError, match="extends past"):
        prepare_fixed_clip(entry, num_frames=30, fps=10.0, height=32, width=32)
    with pytest.raises(ValueError, match="fps"):
        decode_video(dict(frames_path=entry["frames_path"]))


def test_native_clip_trims_to_4k_plus_1(tmp_path):
    entry, _ = _npy(tmp_path, t=23)
    rgb, clip = prepare_native_clip(entry)
    assert rgb.shape[0] == 21 and clip["num_frames"] == 21
    assert wan_latent_shape(21, 48, 64) == (16, 6, 6, 8)
    bad, _ = _npy(tmp_path, t=9, h=40)
    with pytest.raises(ValueError, match="divisible by 16"):
        prepare_native_clip(bad)


def test_qwen_sampling_and_patches(tmp_path):
    assert qwen_frame_indices(21, 8).tolist() == [0, 3, 6, 9, 11, 14, 17, 20]
    assert len(qwen_frame_indices(21, 7)) == 6
    entry, _ = _npy(tmp_path, t=21, h=64, w=64)
    rgb, _ = prepare_native_clip(entry)
    patches, grid, idx = qwen_video_patches(rgb, 4, min_pixels=64 * 64, max_pixels=64 * 64)
    assert grid == (2, 4, 4) and patches.shape == (32, 1536) and len(idx) == 4
