"""Video clip transforms (reference: ospnext/data/utils/transforms.py:14-708).

Clips are tensors [T, C, H, W].  The module is organised in three layers:

* size rules — pure functions of (h, w) that decide a target size or crop box
  (long-side / short-side fit, max-area fit, stride crop, aspect-ratio filter);
* clip operations — crop, flip, resize, centre crops, resize-then-crop-to-fill;
* transform objects — small callables configured once and applied per clip
  (what the data pipelines compose), with the reference's class names.

The Wan pipeline uses ``CenterCropResizeVideo`` (short-side fit with bicubic antialiased
resize, then centre crop), ``ToTensorAfterResize``, ``AENorm`` and ``TemporalRandomCrop``.
"""
from __future__ import annotations

import math
import numbers
import random
from typing import Dict, Optional, Sequence, Tuple, Union

import numpy as np
import torch
import torch.nn.functional as F

Size = Tuple[int, int]


# ---------------------------------------------------------------------------- size rules

def fit_long_side(h: int, w: int, size: Size, skip_low_resolution: bool = False) -> Size:
    """Scale so the clip fits inside ``size`` = (H, W) with its limiting side equal to the
    target (the other side rounded up); small clips unchanged if ``skip_low_resolution``."""
    H, W = size
    if skip_low_resolution and h <= H and w <= W:
        return h, w
    if h * W > H * w:                       # relatively taller than the target: height limits
        return H, math.ceil(H / h * w)
    return math.ceil(W / w * h), W


def fit_short_side(h: int, w: int, size: Size, skip_low_resolution: bool = False) -> Size:
    """Scale so the clip covers ``size`` = (H, W) (the non-limiting side rounded up)."""
    H, W = size
    if skip_low_resolution and h <= H and w <= W:
        return h, w
    if h * W < H * w:                       # relatively wider: match the height, overflow in width
        return H, math.ceil(H / h * w)
    return math.ceil(W / w * h), W


def fit_max_area(h: int, w: int, max_hxw: int) -> Size:
    """Shrink (never enlarge) to at most ``max_hxw`` pixels keeping the aspect ratio."""
    if h * w <= max_hxw:
        return h, w
    s = float(np.sqrt(max_hxw / (h * w)))
    return int(h * s), int(w * s)


def stride_crop_box(h: int, w: int, stride: int) -> Tuple[int, int, int, int]:
    """Centred (top, left, height, width) box with both sides multiples of ``stride``."""
    th, tw = h // stride * stride, w // stride * stride
    return (h - th) // 2, (w - tw) // 2, th, tw


def filter_resolution(h, w, max_h_div_w_ratio=17 / 16, min_h_div_w_ratio=8 / 16) -> bool:
    """Keep clips whose aspect ratio h / w lies in [min, max]."""
    return min_h_div_w_ratio <= h / w <= max_h_div_w_ratio


def calculate_statistics(data):
    """mean / variance / std / min / max of a list of numbers (None when empty)."""
    if len(data) == 0:
        return None
    a = np.asarray(data)
    return {"mean": a.mean(), "variance": a.var(), "std_dev": a.std(), "min": a.min(), "max": a.max()}


# the reference's names for the size rules
longsideresize = fit_long_side
shortsideresize = fit_short_side
maxhwresize = fit_max_area
get_params = stride_crop_box


# ---------------------------------------------------------------------------- clip operations

def _check_clip(clip):
    if not torch.is_tensor(clip):
        raise TypeError(f"clip should be a tensor, got {type(clip)}")
    if clip.dim() != 4:
        raise ValueError(f"clip should be 4-D [T, C, H, W], got {clip.dim()}-D")
    return clip


def to_tensor(clip):
    """uint8 [T, C, H, W] → float in [0, 1]."""
    _check_clip(clip)
    if clip.dtype != torch.uint8:
        raise TypeError(f"clip should be uint8, got {clip.dtype}")
    return clip.float() / 255.0


def to_tensor_after_resize(clip):
    """Resized float clip in [0, 255] → [0, 1]."""
    return clip.float() / 255.0


def hflip(clip):
    return _check_clip(clip).flip(-1)


def crop(clip, top: int, left: int, height: int, width: int):
    if clip.dim() != 4:
        raise ValueError("clip should be a 4-D tensor")
    return clip[..., top:top + height, left:left + width]


def resize(clip, target_size: Size, interpolation_mode: str, align_corners=False, antialias=False):
    if len(target_size) != 2:
        raise ValueError(f"target size should be (height, width), got {target_size}")
    return F.interpolate(clip, size=tuple(target_size), mode=interpolation_mode, align_corners=align_corners,
                         antialias=antialias)


def resize_scale(clip, target_size: Size, interpolation_mode: str):
    """Scale by target_size[0] / short side (aspect ratio kept)."""
    if len(target_size) != 2:
        raise ValueError(f"target size should be (height, width), got {target_size}")
    s = target_size[0] / min(clip.shape[-2], clip.shape[-1])
    return F.interpolate(clip, scale_factor=s, mode=interpolation_mode, align_corners=False)


def center_crop(clip, crop_size: Size):
    h, w = _check_clip(clip).shape[-2:]
    th, tw = crop_size
    if h < th or w < tw:
        raise ValueError(f"clip {h}x{w} is smaller than the crop {crop_size}")
    return crop(clip, int(round((h - th) / 2.0)), int(round((w - tw) / 2.0)), th, tw)


def center_crop_using_short_edge(clip):
    """Centred square of side min(h, w)."""
    h, w = _check_clip(clip).shape[-2:]
    s = min(h, w)
    return crop(clip, int(round((h - s) / 2.0)) if h > w else 0, int(round((w - s) / 2.0)) if w >= h else 0, s, s)


def center_crop_th_tw(clip, th: int, tw: int, top_crop: bool):
    """Largest box of aspect ratio th : tw, horizontally centred, at the top or centred."""
    h, w = _check_clip(clip).shape[-2:]
    r = th / tw
    nh, nw = (int(w * r), w) if h / w > r else (h, int(h / r))
    return crop(clip, 0 if top_crop else int(round((h - nh) / 2.0)), int(round((w - nw) / 2.0)), nh, nw)


def resize_crop_to_fill(clip, target_size: Size):
    """Bilinear resize so the clip covers target_size, then crop the excess (from the
    start of the overflowing side's centred window)."""
    h, w = _check_clip(clip).shape[-2:]
    th, tw = target_size
    rh, rw = th / h, tw / w
    if rh > rw:
        sh, sw = th, round(w * rh)
        top, left = 0, int(round(sw - tw) / 2.0)
    else:
        sh, sw = round(h * rw), tw
        top, left = int(round(sh - th) / 2.0), 0
    clip = resize(clip, (sh, sw), "bilinear")
    if top + th > clip.shape[-2] or left + tw > clip.shape[-1]:
        raise AssertionError("size mismatch.")
    return crop(clip, top, left, th, tw)


# ---------------------------------------------------------------------------- transform objects

class _Named:
    def __repr__(self) -> str:
        args = ", ".join(f"{k}={v}" for k, v in vars(self).items())
        return f"{type(self).__name__}({args})"


class AENorm(_Named):
    """[0, 1] → [-1, 1] (the VAE's input range)."""

    def __call__(self, clip):
        return 2.0 * clip - 1.0


class ToTensorVideo(_Named):
    def __call__(self, clip):
        return to_tensor(clip)


class ToTensorAfterResize(_Named):
    def __call__(self, clip):
        return to_tensor_after_resize(clip)


class RandomHorizontalFlipVideo(_Named):
    def __init__(self, p: float = 0.5):
        self.p = p

    def __call__(self, clip):
        return hflip(clip) if random.random() < self.p else clip


class SpatialStrideCropVideo(_Named):
    """Centre crop to the largest multiple of ``stride`` in both sides."""

    def __init__(self, stride: int):
        self.stride = stride

    def __call__(self, clip):
        return crop(clip, *stride_crop_box(clip.shape[-2], clip.shape[-1], self.stride))


class _Resizer(_Named):
    def __init__(self, interpolation_mode="bilinear", align_corners=False, antialias=False):
        self.interpolation_mode = interpolation_mode
        self.align_corners = align_corners
        self.antialias = antialias

    def _resize_to(self, clip, hw: Size):
        if tuple(hw) == tuple(clip.shape[-2:]):
            return clip
        return resize(clip, hw, self.interpolation_mode, self.align_corners, self.antialias)


class LongSideResizeVideo(_Resizer):
    """Fit inside ``size`` (see :func:`fit_long_side`)."""

    def __init__(self, size, skip_low_resolution=False, interpolation_mode="bilinear", align_corners=False,
                 antialias=False):
        super().__init__(interpolation_mode, align_corners, antialias)
        self.size = size
        self.skip_low_resolution = skip_low_resolution

    def __call__(self, clip):
        h, w = clip.shape[-2:]
        return self._resize_to(clip, fit_long_side(h, w, self.size, self.skip_low_resolution))


class MaxHWResizeVideo(_Resizer):
    """Shrink to at most ``transform_size['max_hxw']`` pixels."""

    def __init__(self, transform_size=None, interpolation_mode="bilinear", align_corners=False, antialias=False):
        if not transform_size or "max_hxw" not in transform_size:
            raise ValueError("Missing required param: max_hxw in data transform.")
        super().__init__(interpolation_mode, align_corners, antialias)
        self.max_hxw = transform_size["max_hxw"]

    def __call__(self, clip):
        h, w = clip.shape[-2:]
        return self._resize_to(clip, fit_max_area(h, w, self.max_hxw))


class CenterCropResizeVideo(_Resizer):
    """Cover ``transform_size`` = (H, W) (short-side fit), then centre crop to it."""

    def __init__(self, transform_size=None, interpolation_mode="bilinear", align_corners=False, antialias=False):
        super().__init__(interpolation_mode, align_corners, antialias)
        self.size = tuple(transform_size)

    def __call__(self, clip):
        h, w = clip.shape[-2:]
        clip = resize(clip, fit_short_side(h, w, self.size), self.interpolation_mode, self.align_corners,
                      self.antialias)
        return center_crop(clip, self.size)


class ResizeVideo(_Resizer):
    """Resize by one of four rules: ``resize`` (fixed size), ``longside``, ``shortside``,
    ``hxw`` (max area).  ``transform_size`` may be a dict with max_height / max_width /
    max_hxw."""

    def __init__(self, transform_size="auto", interpolation_mode="bilinear", skip_low_resolution=False,
                 align_corners=False, antialias=False, mode="resize"):
        super().__init__(interpolation_mode, align_corners, antialias)
        if mode == "hxw":
            self.transform_size = transform_size["max_hxw"] if isinstance(transform_size, dict) else transform_size
        elif mode in ("resize", "longside", "shortside"):
            self.transform_size = ((transform_size["max_height"], transform_size["max_width"])
                                   if isinstance(transform_size, dict) else transform_size)
        else:
            raise NotImplementedError(f"ResizeVideo mode {mode!r}: use resize / longside / shortside / hxw")
        self.mode = mode
        self.skip_low_resolution = skip_low_resolution

    def target(self, h: int, w: int) -> Size:
        if self.mode == "hxw":
            return fit_max_area(h, w, self.transform_size)
        if self.mode == "longside":
            return fit_long_side(h, w, self.transform_size, self.skip_low_resolution)
        if self.mode == "shortside":
            return fit_short_side(h, w, self.transform_size, self.skip_low_resolution)
        return tuple(self.transform_size)

    def __call__(self, clip):
        return self._resize_to(clip, self.target(*clip.shape[-2:]))


class UCFCenterCropVideo(_Named):
    """Scale the short side to size[0], then centre crop to ``size``."""

    def __init__(self, size, interpolation_mode="bilinear"):
        if isinstance(size, (list, tuple)):
            if len(size) != 2:
                raise ValueError(f"size should be (height, width), got {size}")
            self.size = tuple(size)
        else:
            self.size = (size, size)
        self.interpolation_mode = interpolation_mode

    def __call__(self, clip):
        return center_crop(resize_scale(clip, self.size, self.interpolation_mode), self.size)


class _SizeCrop(_Named):
    def __init__(self, size):
        self.size = (int(size), int(size)) if isinstance(size, numbers.Number) else size


class ResizeCrop(_SizeCrop):
    def __call__(self, clip):
        return resize_crop_to_fill(clip, self.size)


class ResizeCropToFill(_Named):
    def __init__(self, size=256):
        self.size = size

    def __call__(self, clip):
        return resize_crop_to_fill(clip, self.size)


class RandomSizedCrop(_SizeCrop):
    """Random crop with height and width drawn from [size[0], size[1]], multiples of 8."""

    def get_params(self, clip, multiples_of: int = 8):
        h, w = clip.shape[-2:]
        th = random.randint(self.size[0], self.size[1])
        tw = random.randint(self.size[0], self.size[1])
        th, tw = th - th % multiples_of, tw - tw % multiples_of
        if h < th:
            th = h - h % multiples_of
        if w < tw:
            tw = w - w % multiples_of
        if (th, tw) == (h, w):
            return 0, 0, h, w
        return random.randint(0, h - th), random.randint(0, w - tw), th, tw

    def __call__(self, clip):
        return crop(clip, *self.get_params(clip))


class TemporalRandomCrop(_Named):
    """Frame window [begin, end) of ``size`` frames: from the start, or at a random start in
    [0, total − size − 1]."""

    def __init__(self, size: int, force_cut_video_from_start: bool = False):
        self.size = size
        self.force_cut_video_from_start = force_cut_video_from_start

    def __call__(self, total_frames: int):
        begin = 0 if self.force_cut_video_from_start else random.randint(0, max(0, total_frames - self.size - 1))
        return begin, min(begin + self.size, total_frames)


class Expand2Square(_Named):
    """Pad a PIL image to a square with the mean colour (images are centred)."""

    def __init__(self, mean: Sequence[float]):
        self.background_color = tuple(int(x * 255) for x in mean)

    def __call__(self, pil_img):
        from PIL import Image
        w, h = pil_img.size
        if w == h:
            return pil_img
        side = max(w, h)
        out = Image.new(pil_img.mode, (side, side), self.background_color)
        out.paste(pil_img, ((side - w) // 2, (side - h) // 2))
        return out


class Compose(_Named):
    def __init__(self, fs):
        self.fs = list(fs)

    def __call__(self, x):
        for f in self.fs:
            x = f(x)
        return x


def center_crop_resize(video: torch.Tensor, size, interpolation="bicubic", antialias=True) -> torch.Tensor:
    """The Wan pipeline's spatial transform on a [T, C, H, W] clip (float output)."""
    return CenterCropResizeVideo(size, interpolation, False, antialias)(video.float())
