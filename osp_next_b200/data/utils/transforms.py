"""Video transforms (reference: ospnext/data/utils/transforms.py:14-708, the subset the
Wan pipeline uses): centre-crop-resize (bicubic, antialias), uint8→float, [-1,1]
normalisation, random / start temporal crop, flips, aspect-ratio filter."""
from __future__ import annotations

import random

import torch
import torch.nn.functional as F


def center_crop_resize(video: torch.Tensor, size, interpolation="bicubic", antialias=True) -> torch.Tensor:
    """[T,C,H,W] → crop to the target aspect ratio around the centre, then resize."""
    th, tw = size
    T, C, H, W = video.shape
    if H / W > th / tw:
        nh, nw = int(round(W * th / tw)), W
    else:
        nh, nw = H, int(round(H * tw / th))
    y0, x0 = (H - nh) // 2, (W - nw) // 2
    v = video[:, :, y0:y0 + nh, x0:x0 + nw].float()
    return F.interpolate(v, size=(th, tw), mode=interpolation, align_corners=False, antialias=antialias)


class CenterCropResizeVideo:
    def __init__(self, size, interpolation_mode="bicubic", align_corners=False, antialias=True):
        self.size, self.mode, self.antialias = size, interpolation_mode, antialias

    def __call__(self, v):
        return center_crop_resize(v, self.size, self.mode, self.antialias)


class ToTensorAfterResize:
    def __call__(self, v):
        return v.float() / 255.0


class AENorm:
    """[0,1] → [-1,1]."""

    def __call__(self, v):
        return 2.0 * v - 1.0


class TemporalRandomCrop:
    def __init__(self, size: int, force_cut_video_from_start: bool = False):
        self.size = size
        self.from_start = force_cut_video_from_start

    def __call__(self, total: int):
        if self.from_start:
            return 0, min(self.size, total)
        b = random.randint(0, max(0, total - self.size))
        return b, min(b + self.size, total)


class RandomHorizontalFlipVideo:
    def __init__(self, p: float = 0.5):
        self.p = p

    def __call__(self, v):
        return v.flip(-1) if random.random() < self.p else v


def filter_resolution(h, w, max_h_div_w_ratio=17 / 16, min_h_div_w_ratio=8 / 16) -> bool:
    r = h / w
    return min_h_div_w_ratio <= r <= max_h_div_w_ratio


class Compose:
    def __init__(self, fs):
        self.fs = fs

    def __call__(self, x):
        for f in self.fs:
            x = f(x)
        return x
