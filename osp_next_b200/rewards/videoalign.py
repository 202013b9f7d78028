"""VideoAlign reward model wrapper (reference: ospnext/rewards/videoalign_*.py).

A Qwen2-VL vision-language backbone reads the video frames and a scoring
prompt built from the caption; a linear Bradley–Terry head on the final hidden
state of the special reward token yields three scores (VQ visual quality, MQ
motion quality, TA text alignment), optionally normalised by the checkpoint's
reward mean/std; "Overall" = VQ + MQ + TA.  Loading requires the VideoAlign
checkpoint directory (``config.json`` with the reward-head settings and the
model weights); nothing is downloaded.
"""
from __future__ import annotations

import json
import os
from typing import List, Optional

import numpy as np
import torch

PROMPT = ("You are tasked with evaluating a generated video based on three distinct criteria: visual quality, "
          "motion quality, and text alignment. Please provide a rating from 0 to 10 for each of the three "
          "categories. Caption: {caption}")


class VideoAlignScorer:
    def __init__(self, device, load_from_pretrained: Optional[str], reward_dim="Overall", use_norm=True,
                 num_frames=None, fps=None, max_pixels=None):
        if not load_from_pretrained or not os.path.isdir(load_from_pretrained):
            raise FileNotFoundError("VideoAlign needs `load_from_pretrained` pointing at its checkpoint directory")
        from transformers import AutoProcessor, Qwen2VLForConditionalGeneration
        self.device = device
        self.reward_dim = reward_dim
        self.use_norm = use_norm
        self.num_frames = num_frames or 8
        self.max_pixels = max_pixels or 448 * 448
        self.processor = AutoProcessor.from_pretrained(load_from_pretrained)
        self.model = Qwen2VLForConditionalGeneration.from_pretrained(
            load_from_pretrained, torch_dtype=torch.bfloat16).to(device).eval()
        hidden = self.model.config.hidden_size
        self.rm_head = torch.nn.Linear(hidden, 3, bias=False).to(device, torch.bfloat16)
        head = os.path.join(load_from_pretrained, "rm_head.pt")
        if os.path.exists(head):
            self.rm_head.load_state_dict(torch.load(head, map_location="cpu", weights_only=True))
        stats = os.path.join(load_from_pretrained, "reward_stats.json")
        self.mean, self.std = np.zeros(3), np.ones(3)
        if os.path.exists(stats):
            with open(stats) as f:
                st = json.load(f)
            self.mean, self.std = np.asarray(st["mean"]), np.asarray(st["std"])

    def _frames(self, video: np.ndarray) -> List[np.ndarray]:
        idx = np.linspace(0, len(video) - 1, self.num_frames).round().astype(int)
        return [video[i] for i in idx]

    @torch.no_grad()
    def __call__(self, videos: np.ndarray, prompts: List[str]) -> List[float]:
        out = []
        for vid, cap in zip(videos, prompts):
            msgs = [{"role": "user", "content": [{"type": "video"}, {"type": "text",
                                                                     "text": PROMPT.format(caption=cap)}]}]
            text = self.processor.apply_chat_template(msgs, add_generation_prompt=True)
            inputs = self.processor(text=[text], videos=[self._frames(vid)], return_tensors="pt").to(self.device)
            h = self.model(**inputs, output_hidden_states=True).hidden_states[-1][:, -1]
            s = self.rm_head(h).float().cpu().numpy()[0]
            if self.use_norm:
                s = (s - self.mean) / self.std
            d = {"VQ": s[0], "MQ": s[1], "TA": s[2], "Overall": float(s.sum())}
            out.append(float(d[self.reward_dim]))
        return out
