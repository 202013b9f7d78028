"""Wan data processors (reference: ospnext/data/utils/wan_utils.py:12-320).

* ``WanTextProcessor``: caption cleaning (URL/HTML removal, lower-case,
  whitespace) then tokenisation padded to ``model_max_length`` with the mask.
* ``WanVideoFilter``: drops samples without caption / resolution, with the
  wrong aspect ratio, too small, too long, below the training fps, outside the
  motion range, or with fewer usable frames than ``sample_num_frames``.
* ``WanVideoProcessor``: fps resampling (``train_fps``) or fixed stride, random
  temporal crop, optional spatial crop, centre-crop-resize (bicubic), [-1, 1],
  returned as ``[C, T, H, W]``.
"""
from __future__ import annotations

import html
import json
import math
import re
import urllib.parse as ul
from typing import Dict, List, Optional

import numpy as np
import torch

from .transforms import (AENorm, CenterCropResizeVideo, Compose, TemporalRandomCrop, ToTensorAfterResize,
                         filter_resolution)
from .video_io import video_reader_contextmanager

_URL = re.compile(r"\b((?:https?:(?:/{1,3}|[a-zA-Z0-9%])|[a-zA-Z0-9.\-]+[.](?:com|co|ru|net|org|edu|gov|it)"
                  r"[\w/-]*\b/?(?!@)))")


def clean_caption(caption: str) -> str:
    c = ul.unquote_plus(str(caption)).strip().lower()
    c = re.sub("<person>", "person", c)
    c = _URL.sub("", c)
    c = html.unescape(html.unescape(c))
    c = re.sub(r"<[^>]+>", " ", c)
    c = re.sub(r"@[\w\d]+\b", "", c)
    c = re.sub(r"\s+", " ", c)
    return c.strip()


class WanTextProcessor:
    def __init__(self, tokenizer, model_max_length=512, return_prompt_mask=True, use_clean_caption=True,
                 enable_text_preprocessing=True, padding_type="max_length"):
        self.tokenizer = tokenizer
        self.model_max_length = model_max_length
        self.return_prompt_mask = return_prompt_mask
        self.use_clean_caption = use_clean_caption
        self.enable_text_preprocessing = enable_text_preprocessing
        self.padding_type = padding_type

    def __call__(self, text: str):
        if self.enable_text_preprocessing:
            text = clean_caption(text) if self.use_clean_caption else text.lower().strip()
        if self.tokenizer is None:               # tokenizer-less synthetic mode: EOS only
            ids = torch.zeros(1, self.model_max_length, dtype=torch.long)
            mask = torch.zeros(1, self.model_max_length, dtype=torch.long)
            ids[0, 0], mask[0, 0] = 1, 1
            return ids, (mask if self.return_prompt_mask else None)
        out = self.tokenizer(text, max_length=self.model_max_length, padding=self.padding_type, truncation=True,
                             add_special_tokens=True, return_tensors="pt")
        return out.input_ids, (out.attention_mask if self.return_prompt_mask else None)


def read_ann_txt(path: str) -> List[Dict]:
    """Annotation list: a JSON file (list of records) or JSONL."""
    with open(path, encoding="utf-8") as f:
        head = f.read(1)
        f.seek(0)
        if head == "[":
            return json.load(f)
        return [json.loads(l) for l in f if l.strip()]


class WanVideoFilter:
    def __init__(self, ann_txt_path=None, sample_height=480, sample_width=832, sample_num_frames=49, train_fps=16,
                 sample_stride=None, min_hxw=480 * 832, too_long_factor=5.0, max_h_div_w_ratio=2.0,
                 min_h_div_w_ratio=0.5, max_motion_value=1.0, min_motion_value=0.0, data_samples=None, **kw):
        self.data_samples = data_samples if data_samples is not None else (read_ann_txt(ann_txt_path)
                                                                          if ann_txt_path else [])
        self.h, self.w, self.f = sample_height, sample_width, sample_num_frames
        self.train_fps, self.sample_stride = train_fps, sample_stride
        if train_fps is None and sample_stride is None:
            raise ValueError("Must specify either train_fps or sample_stride")
        self.min_hxw, self.too_long = min_hxw, too_long_factor
        self.max_r, self.min_r = max_h_div_w_ratio, min_h_div_w_ratio
        self.max_m, self.min_m = max_motion_value, min_motion_value
        self.stats = {}

    def _interval(self, fps):
        if self.train_fps is not None:
            return 1.0 if abs(fps - self.train_fps) < 0.1 else fps / self.train_fps
        return self.sample_stride

    def filter_data_samples_force_shape(self, data_samples=None) -> List[Dict]:
        data = self.data_samples if data_samples is None else data_samples
        st = dict.fromkeys(["no_cap", "no_resolution", "aspect_mismatch", "res_too_small", "too_long",
                            "fps_too_low", "too_fast", "too_slow", "too_short"], 0)
        out = []
        for s in data:
            if s.get("cap") is None:
                st["no_cap"] += 1
                continue
            res = s.get("resolution") or {}
            hh, ww = res.get("height"), res.get("width")
            if not hh or not ww or hh <= 0 or ww <= 0:
                st["no_resolution"] += 1
                continue
            if not filter_resolution(hh, ww, self.max_r, self.min_r):
                st["aspect_mismatch"] += 1
                continue
            tr, cr = self.h / self.w, hh / ww
            if hh * ww < math.ceil(self.min_hxw * max(cr / tr, tr / cr)):
                st["res_too_small"] += 1
                continue
            fps = s.get("fps", 24)
            ref_fps = self.train_fps or fps
            if s["num_frames"] > self.too_long * (self.f * fps / ref_fps):
                st["too_long"] += 1
                continue
            itv = self._interval(fps)
            if self.train_fps is not None and itv < 1.0:
                st["fps_too_low"] += 1
                continue
            mv = s.get("motion", 0.0)
            if mv < self.min_m:
                st["too_fast"] += 1
                continue
            if mv > self.max_m:
                st["too_slow"] += 1
                continue
            start = s.get("cut", [0])[0]
            s["start_frame_idx"] = start
            if len(np.arange(start, start + s["num_frames"], itv)) < self.f:
                st["too_short"] += 1
                continue
            out.append(s)
        self.stats = dict(st, before=len(data), after=len(out))
        return out


class WanVideoProcessor:
    def __init__(self, sample_height=480, sample_width=832, sample_num_frames=49, train_fps=None, sample_stride=None,
                 force_cut_video_from_start=False):
        self.h, self.w, self.f = sample_height, sample_width, sample_num_frames
        self.train_fps, self.sample_stride = train_fps, sample_stride
        if train_fps is None and sample_stride is None:
            raise ValueError("Must specify either train_fps or sample_stride")
        self.transforms = Compose([CenterCropResizeVideo((self.h, self.w), interpolation_mode="bicubic",
                                                         align_corners=False, antialias=True),
                                   ToTensorAfterResize(), AENorm()])
        self.temporal_sample = TemporalRandomCrop(self.f, force_cut_video_from_start)

    def read_one_sample(self, path, meta: Optional[Dict] = None) -> torch.Tensor:
        meta = meta or {}
        with video_reader_contextmanager(path) as r:
            fps = r.get_video_fps() if r.get_video_fps() > 0 else 30.0
            if abs(fps - meta.get("fps", fps)) > 0.1:
                raise ValueError(f"fps mismatch: {fps} vs {meta.get('fps')} ({path})")
            total = meta.get("num_frames", r.get_num_frames())
            start = meta.get("start_frame_idx", 0)
            itv = (1.0 if abs(fps - self.train_fps) < 0.1 else fps / self.train_fps) if self.train_fps else \
                self.sample_stride
            idx = np.arange(start, start + total, itv).astype(int)
            if len(idx) < self.f:
                raise ValueError(f"need {self.f} frames, got {len(idx)} ({path})")
            b, e = self.temporal_sample(len(idx))
            v = r.get_batch(idx[b:e])
            crop = meta.get("crop")
            if crop and crop[0] is not None:
                sx, ex, sy, ey = crop
                v = v[:, :, sy:ey, sx:ex]
        return v

    def process_one_sample(self, v: torch.Tensor) -> torch.Tensor:
        v = self.transforms(v).permute(1, 0, 2, 3)
        if tuple(v.shape[1:]) != (self.f, self.h, self.w):
            raise ValueError(f"bad sample shape {tuple(v.shape)}")
        return v

    def __call__(self, path, meta=None, need_processing=True):
        v = self.read_one_sample(path, meta)
        return self.process_one_sample(v) if need_processing else v
