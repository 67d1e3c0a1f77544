"""Evaluation outputs: decoded visuals to files, and reference scores of a case.

* ``save_visual(pixels, path)``: ``pixels`` uint8 / float ``[T, H, W, 3]`` (or ``[H, W, 3]``) in
  [0, 255] or [0, 1]. One frame -> PNG; several -> MP4 (H.264 through PyAV when it is installed,
  as the reference writes them, ``evaluations/sampling.py:49-59``), otherwise an animated WebP at
  the same frame rate. Returns the written path.
* ``latent_preview(latent)``: an RGB preview of a latent ``[C, T, H, W]`` (channels 0-2, each
  min/max scaled) for runs without a VAE decoder, so a report always shows something.
* ``reference_scores(model, batch)``: teacher-forced scores of a case's reference targets: the
  mean text NLL over its supervised text positions, and the flow-matching MSE of its generation
  targets at fixed noise and flow times (the deterministic preparation of the batch), i.e. the
  training losses evaluated without gradient (reference ``evaluations/sampling.py:62-140``).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch


def _frames(pixels):
    array = pixels.detach().float().cpu().numpy() if isinstance(pixels, torch.Tensor) else np.asarray(pixels)
    if array.ndim == 3:
        array = array[None]
    if array.ndim != 4 or array.shape[-1] != 3:
        raise ValueError(f"expected [T, H, W, 3] pixels, got {array.shape}")
    if array.dtype != np.uint8:
        scale = 255.0 if array.max() <= 1.0 + 1e-6 else 1.0
        array = np.clip(np.rint(array * scale), 0, 255).astype(np.uint8)
    return array


def save_visual(pixels, path, fps=16):
    from PIL import Image
    frames = _frames(pixels)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    if len(frames) == 1:
        out = path.with_suffix(".png")
        Image.fromarray(frames[0]).save(out)
        return out
    try:
        import av
    except ImportError:
        av = None
    if av is not None:
        out = path.with_suffix(".mp4")
        with av.open(str(out), mode="w") as container:
            stream = container.add_stream("libx264", rate=fps)
            stream.width, stream.height = frames.shape[2] - frames.shape[2] % 2, frames.shape[1] - frames.shape[1] % 2
            stream.pix_fmt = "yuv420p"
            for frame in frames:
                picture = av.VideoFrame.from_ndarray(frame[: stream.height, : stream.width], format="rgb24")
                for packet in stream.encode(picture):
                    container.mux(packet)
            for packet in stream.encode():
                container.mux(packet)
        return out
    out = path.with_suffix(".webp")
    images = [Image.fromarray(f) for f in frames]
    images[0].save(out, save_all=True, append_images=images[1:], duration=int(1000 / fps), loop=0, lossless=True)
    return out


def latent_preview(latent):
    """``[C, T, H, W]`` latent -> uint8 ``[T, H, W, 3]`` from channels 0-2 (min/max scaled each)."""
    x = latent[:3].detach().float().cpu()
    lo = x.amin(dim=(1, 2, 3), keepdim=True)
    hi = x.amax(dim=(1, 2, 3), keepdim=True)
    x = (x - lo) / (hi - lo).clamp_min(1e-6)
    return (x.permute(1, 2, 3, 0) * 255).round().to(torch.uint8).numpy()


@torch.no_grad()
def reference_scores(model, batch):
    """``{"text_nll": mean NLL per supervised token or None, "flow_mse": weighted flow MSE or None}``."""
    out = model(batch, compute_image_loss=batch.generation is not None)
    text = out.get("text_loss")
    image = out.get("image_loss")
    has_text = int(batch.text_indices.numel()) > 0
    return dict(text_nll=float(text) if has_text and text is not None else None,
                flow_mse=float(image) if image is not None and batch.generation is not None else None,
                text_tokens=int(batch.text_indices.numel()),
                generation_targets=int(batch.generation_image_count) if batch.generation is not None else 0)
