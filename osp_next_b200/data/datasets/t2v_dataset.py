"""Text-to-video datasets (reference: ospnext/data/datasets/t2v_dataset.py:20-178).

* ``WanT2VDataset``: metadata store (LMDB or JSONL) → caption (10 % dropped to
  "" for CFG) + video clip decoded, fps-resampled, centre-cropped/resized,
  scaled to [-1, 1]; each item is loaded in a one-thread executor with a
  timeout and a failing item is replaced by a random other index.
* ``T2VRandomDataset``: random video of the configured size and an empty prompt.
* ``T2VRandomLatentDataset`` (addition): random VAE latents and T5-shaped
  embeddings, so training can be benchmarked without the frozen encoders.
"""
from __future__ import annotations

import copy
import random
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from ...utils.constant import PROMPT_IDS, PROMPT_MASK, VIDEO
from ..utils.meta_store import open_meta_reader
from ..utils.wan_utils import WanTextProcessor, WanVideoProcessor
from .base_dataset import BaseDataset

T2VOutputData = {PROMPT_IDS: None, PROMPT_MASK: None, VIDEO: None}


def _tokenizer(path):
    if path is None:
        return None
    from ...models.tokenizers import load_tokenizer
    return load_tokenizer(path)


class WanT2VDataset(BaseDataset):
    def __init__(self, metafile_or_dir_path, text_tokenizer_path=None, sample_height=480, sample_width=832,
                 sample_num_frames=49, train_fps=16, sample_stride=None, text_drop_ratio=0.1, text_max_length=512,
                 return_prompt_mask=True, timeout=600, **kwargs):
        self.metafile_or_dir_path = metafile_or_dir_path
        self._reader = None
        self.data_length = len(open_meta_reader(metafile_or_dir_path))
        if train_fps is None and sample_stride is None:
            raise ValueError("Must specify either train_fps or sample_stride")
        self.text_drop_ratio = text_drop_ratio
        self.text_processor = WanTextProcessor(_tokenizer(text_tokenizer_path), text_max_length, return_prompt_mask)
        self.video_processor = WanVideoProcessor(sample_height, sample_width, sample_num_frames, train_fps,
                                                 sample_stride)
        self._executor = None
        self.timeout = timeout

    @property
    def reader(self):
        if self._reader is None:                      # opened lazily inside each worker
            self._reader = open_meta_reader(self.metafile_or_dir_path)
        return self._reader

    @property
    def executor(self):
        if self._executor is None:
            self._executor = ThreadPoolExecutor(max_workers=1)
        return self._executor

    def __len__(self):
        return self.data_length

    def __getitem__(self, index):
        for _ in range(32):
            try:
                return self.executor.submit(self.getitem, index).result(timeout=self.timeout)
            except Exception as e:  # corrupt / slow sample: take another one
                print(f"[WanT2VDataset] item {index} failed: {e}")
                index = np.random.randint(0, max(1, len(self) - 1))
        raise RuntimeError("too many consecutive failing samples")

    def getitem(self, index):
        ex = copy.deepcopy(T2VOutputData)
        meta = self.reader.getitem(index)
        ex[PROMPT_IDS], ex[PROMPT_MASK] = self.get_text_data(meta["cap"])
        ex[VIDEO] = self.video_processor(meta["path"], meta)
        return ex

    def get_text_data(self, text):
        if isinstance(text, list):
            text = random.choice(text)
        if random.random() < self.text_drop_ratio:
            text = ""
        return self.text_processor(text)


class T2VRandomDataset(BaseDataset):
    def __init__(self, text_tokenizer_path=None, sample_height=480, sample_width=832, sample_num_frames=49,
                 text_max_length=512, return_prompt_mask=True, **kwargs):
        self.h, self.w, self.f = sample_height, sample_width, sample_num_frames
        self.text_processor = WanTextProcessor(_tokenizer(text_tokenizer_path), text_max_length, return_prompt_mask)

    def __len__(self):
        return 1000000

    def __getitem__(self, index):
        ex = copy.deepcopy(T2VOutputData)
        ex[PROMPT_IDS], ex[PROMPT_MASK] = self.text_processor("")
        ex[VIDEO] = torch.randn(3, self.f, self.h, self.w)
        return ex


class T2VRandomLatentDataset(BaseDataset):
    """Latent-space synthetic data: {"latents": [16, T, H/8, W/8], "text": [L, 4096]} ~ N(0, 1)."""

    def __init__(self, sample_height=768, sample_width=1280, sample_num_frames=81, text_max_length=512,
                 text_dim=4096, latent_channels=16, **kwargs):
        self.shape = (latent_channels, (sample_num_frames - 1) // 4 + 1, sample_height // 8, sample_width // 8)
        self.text_shape = (text_max_length, text_dim)

    def __len__(self):
        return 1000000

    def __getitem__(self, index):
        g = torch.Generator().manual_seed(int(index))
        return {"latents": torch.randn(self.shape, generator=g), "text": torch.randn(self.text_shape, generator=g)}
