"""Video decoding and clip preparation for the understanding tower and the Wan renderer.

* ``decode_video(entry)`` returns uint8 frames ``[T, H, W, 3]``, their presentation times (s) and
  the source sha256. ``.npy`` frame arrays need an explicit ``fps``; other containers decode with
  PyAV when it is installed (it is optional; the error names it otherwise). Times must increase.
* ``prepare_fixed_clip`` picks ``num_frames`` frames at ``fps`` from ``start_seconds`` by nearest
  timestamp, resizes with bicubic (antialiased) interpolation to cover ``height x width`` and
  centre-crops: the fixed-geometry training clip.
* ``prepare_native_clip`` keeps the decoded pixels and trims only the tail so the frame count is
  4k + 1 (Wan's causal VAE maps 4k + 1 frames to k + 1 latent frames); H and W must already be
  multiples of 16.
* ``qwen_frame_indices`` spreads ``count`` frames evenly over a clip (an even count: the tower's
  temporal patch is 2), ``qwen_video_patches`` turns them into tower patches and the grid.
* ``wan_latent_shape`` is the latent geometry ``[16, 1 + (T - 1)/4, H/8, W/8]`` of a clip.

Reference: ``data/video.py:11-220`` (the PyAV path and the fixed/native preparation rules).
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F


def decode_video(entry):
    path = Path(entry.get("frames_path") or entry.get("path") or "")
    if not path.is_file():
        raise FileNotFoundError(f"video not found: {path}")
    if path.suffix == ".npy":
        frames = np.load(path, allow_pickle=False)
        fps = entry.get("fps")
        if fps is None or float(fps) <= 0:
            raise ValueError("NPY frames need an explicit positive fps")
        times = np.arange(len(frames), dtype=np.float64) / float(fps)
    else:
        try:
            import av
        except ImportError as error:
            raise ImportError("decoding video containers needs PyAV (pip install av)") from error
        with av.open(str(path)) as container:
            stream = container.streams.video[0]
            decoded = [(f.to_ndarray(format="rgb24"), float(f.time)) for f in container.decode(stream)]
        if not decoded:
            raise ValueError(f"empty video: {path}")
        frames = np.stack([f for f, _ in decoded])
        times = np.array([t for _, t in decoded]) - decoded[0][1]
    if frames.ndim != 4 or frames.shape[-1] != 3 or frames.dtype != np.uint8:
        raise ValueError("decoded frames must be uint8 [T, H, W, 3]")
    if len(times) < 2 or not np.isfinite(times).all() or not (np.diff(times) > 0).all():
        raise ValueError("a video needs at least two frames with increasing timestamps")
    digest = hashlib.sha256(path.read_bytes()).hexdigest()
    return frames, times, digest


def _cover_crop(rgb, height, width):
    """Bicubic resize so the frame covers (height, width), then centre crop; uint8 [T, 3, h, w]."""
    x = rgb.float()
    scale = max(height / x.shape[2], width / x.shape[3])
    size = (max(height, round(x.shape[2] * scale)), max(width, round(x.shape[3] * scale)))
    x = F.interpolate(x, size=size, mode="bicubic", align_corners=False, antialias=True).clamp(0, 255)
    y0, x0 = (size[0] - height) // 2, (size[1] - width) // 2
    return x[:, :, y0:y0 + height, x0:x0 + width].round().to(torch.uint8)


def prepare_fixed_clip(entry, num_frames, fps, height, width):
    frames, times, digest = decode_video(entry)
    start = float(entry.get("start_seconds", 0.0))
    wanted = start + np.arange(num_frames) / float(fps)
    if wanted[0] < times[0] - 1e-6 or wanted[-1] > times[-1] + 1e-5:
        raise ValueError("the requested clip extends past the source; choose a shorter clip")
    indices = np.abs(times[:, None] - wanted[None]).argmin(0)
    rgb = _cover_crop(torch.from_numpy(frames[indices].copy()).permute(0, 3, 1, 2), height, width)
    clip = dict(source_sha256=digest, frame_indices=indices.tolist(), timestamps=times[indices].tolist(),
                num_frames=int(num_frames), fps=float(fps), height=int(height), width=int(width),
                spatial_transform="bicubic_cover_center_crop")
    return rgb, clip


def prepare_native_clip(entry, expected_num_frames=None):
    if entry.get("start_seconds", 0):
        raise ValueError("native clips use the whole video (start_seconds must be 0)")
    frames, times, digest = decode_video(entry)
    if expected_num_frames is not None:
        if len(frames) != expected_num_frames:
            raise ValueError(f"decoded {len(frames)} frames, expected {expected_num_frames}")
        if (expected_num_frames - 1) % 4:
            raise ValueError("an exact native clip must have 4k + 1 frames")
    if len(frames) < 5:
        raise ValueError("native clips need at least 5 frames")
    t, h, w, _ = frames.shape
    if h % 16 or w % 16:
        raise ValueError("native clips need H and W divisible by 16 (no resize is performed)")
    keep = 1 + 4 * ((t - 1) // 4)
    rgb = torch.from_numpy(frames[:keep].copy()).permute(0, 3, 1, 2)
    clip = dict(source_sha256=digest, frame_indices=list(range(keep)), timestamps=times[:keep].tolist(),
                num_frames=keep, height=h, width=w, spatial_transform="none")
    return rgb, clip


def qwen_frame_indices(num_frames, count):
    count = min(int(count), num_frames)
    count -= count % 2
    if count < 2:
        raise ValueError("the tower needs at least two frames (temporal patch 2)")
    return np.linspace(0, num_frames - 1, count).round().astype(int)


def qwen_video_patches(rgb, count, min_pixels=65536, max_pixels=1048576):
    """uint8 ``[T, 3, H, W]`` -> (tower patches, grid (t, h, w), frame indices)."""
    from .vision import MEAN, STD, patchify, smart_size
    idx = qwen_frame_indices(len(rgb), count)
    h, w = smart_size(rgb.shape[2], rgb.shape[3], min_pixels, max_pixels)
    x = F.interpolate(rgb[idx].float(), size=(h, w), mode="bicubic", align_corners=False, antialias=True)
    x = (x.clamp(0, 255) / 255.0 - torch.tensor(MEAN)[:, None, None]) / torch.tensor(STD)[:, None, None]
    patches, grid = patchify(x)
    return patches, grid, idx


def wan_latent_shape(num_frames, height, width, channels=16):
    if (num_frames - 1) % 4 or height % 8 or width % 8:
        raise ValueError("Wan clips need 4k + 1 frames and H, W divisible by 8")
    return (channels, 1 + (num_frames - 1) // 4, height // 8, width // 8)
