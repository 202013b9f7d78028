"""Inference IO: mp4 writing, video grids, prompt/image lists
(reference: ospnext/utils/infer_utils.py:8-83).

Videos are uint8 ``[T, H, W, C]`` (or a batch ``[B, T, H, W, C]`` / list of them);
mp4 encoding goes through OpenCV (imageio/ffmpeg are not part of this image).
File names follow the reference: ``video_{i}.mp4`` and ``video_grid.mp4``.
"""
from __future__ import annotations

import math
import os
from typing import List, Optional, Sequence, Union

import torch

from ..data.utils.video_io import read_image, save_video

IMAGE_EXTS = (".jpg", ".jpeg", ".png", ".bmp", ".webp", ".tif", ".tiff")


def is_image_file(path: str) -> bool:
    return path.lower().endswith(IMAGE_EXTS)


def save_videos(videos, start_index: int, save_path: str, fps: int):
    """One ``video_{start_index + i}.mp4`` per video of a batch (or one for a single video)."""
    os.makedirs(save_path, exist_ok=True)
    if isinstance(videos, (list, tuple)) or videos.ndim == 5:
        for i, v in enumerate(videos):
            save_video(v, os.path.join(save_path, f"video_{start_index + i}.mp4"), fps=fps)
    elif videos.ndim == 4:
        save_video(videos, os.path.join(save_path, f"video_{start_index}.mp4"), fps=fps)
    else:
        raise ValueError("The video must be in either [b, t, h, w, c] or [t, h, w, c] format.")


def save_video_with_name(video, name: str, save_path: str, fps: int):
    os.makedirs(save_path, exist_ok=True)
    save_video(video, os.path.join(save_path, f"{name}.mp4"), fps=fps)


def make_video_grid(videos: Union[torch.Tensor, Sequence[torch.Tensor]], nrow: Optional[int] = None,
                    padding: int = 1) -> torch.Tensor:
    """Tile ``[B,T,H,W,C]`` uint8 videos into one ``[T, H', W', C]`` grid: ``nrow`` rows
    (default ⌈√B⌉), ⌈B/nrow⌉ columns, cell (r, c) at pixel ((padding+H)·r, (padding+W)·c),
    so black separators of ``padding`` pixels follow every cell (the reference's layout)."""
    if not torch.is_tensor(videos):
        videos = torch.stack(list(videos))
    b, t, h, w, c = videos.shape
    nrow = nrow or math.ceil(math.sqrt(b))
    ncol = math.ceil(b / nrow)
    grid = torch.zeros(t, (padding + h) * nrow + padding, (padding + w) * ncol + padding, c, dtype=torch.uint8)
    for i in range(b):
        r, cc = divmod(i, ncol)
        y, x = (padding + h) * r, (padding + w) * cc
        grid[:, y:y + h, x:x + w] = videos[i].to(torch.uint8).cpu()
    return grid


def save_video_grid(videos, save_path: str, fps: int, nrow: Optional[int] = None):
    os.makedirs(save_path, exist_ok=True)
    save_video(make_video_grid(videos, nrow), os.path.join(save_path, "video_grid.mp4"), fps=fps)


def load_prompts(prompt: str) -> List[str]:
    """A prompt file (one per line) or a literal prompt string."""
    if os.path.exists(prompt):
        with open(prompt, "r") as f:
            return [line.strip() for line in f.readlines()]
    return [prompt]


def _load_image(path: str, layout: str, array_type: str):
    im = read_image(path)                           # uint8 [C,H,W]
    if layout == "HWC":
        im = im.permute(1, 2, 0).contiguous()
    return im.numpy() if array_type == "numpy" else im


def load_images(image: Optional[str] = None, dual_image: bool = False, layout: str = "CHW",
                array_type: str = "torch"):
    """None (text-to-video), one image, or a list file of images (pairs ``a,b`` per
    line when ``dual_image``)."""
    if image is None:
        return None
    if not os.path.exists(image):
        raise FileNotFoundError(f"The image path {image} does not exist")
    if is_image_file(image) and not dual_image:
        return [_load_image(image, layout, array_type)]
    with open(image, "r") as f:
        lines = [ln for ln in f.readlines() if ln.strip()]
    if dual_image:
        out = []
        for ln in lines:
            paths = ln.strip().split(",")
            if len(paths) != 2:
                raise ValueError(f"Each line must contain two paths separated by commas (,). Current line:{ln}")
            out.append([_load_image(p, layout, array_type) for p in paths])
        return out
    return [_load_image(ln.strip(), layout, array_type) for ln in lines]
