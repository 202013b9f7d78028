"""Reward functions for Mix-GRPO (reference: ospnext/rewards/rewards.py:6-107).

``multi_score(device, {"name": weight, …})`` returns ``fn(videos_or_latents,
prompts, metadata) → ({name: scores, "avg": weighted sum}, {})`` like the
reference.  Scores:

* ``videoalign``: the VideoAlign reward model (Qwen2-VL backbone with a
  3-dimensional Bradley–Terry head: VQ, MQ, TA; "Overall" = their sum), see
  :mod:`.videoalign` — needs its checkpoint directory.
* ``latent_mlp`` (addition, used by the RL benchmark): a fixed random-init
  4-layer MLP scoring mean-pooled latents, so RL can run without video decoding
  or a reward checkpoint.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch
import torch.nn as nn


class LatentMLPReward(nn.Module):
    """score = MLP(mean over (t,h,w) of the latent) → scalar, weights fixed by seed."""

    def __init__(self, channels=16, hidden=256, layers=4, seed=0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        dims = [channels] + [hidden] * (layers - 1) + [1]
        mods = []
        for i in range(layers):
            lin = nn.Linear(dims[i], dims[i + 1])
            with torch.no_grad():
                lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) / dims[i] ** 0.5)
                lin.bias.zero_()
            mods += [lin] + ([nn.SiLU()] if i < layers - 1 else [])
        self.net = nn.Sequential(*mods).requires_grad_(False)

    @torch.no_grad()
    def forward(self, latents):
        x = latents.float().mean(dim=tuple(range(2, latents.ndim)))
        return self.net.to(x.device)(x).squeeze(-1)


def latent_mlp_score(device, seed: int = 0, channels: int = 16):
    model = LatentMLPReward(channels=channels, seed=seed).to(device)

    def _fn(latents, prompts, metadata):
        return model(latents.to(device)).cpu().tolist(), {}
    return _fn


def videoalign_score(device, load_from_pretrained=None, load_from_pretrained_step=-1, reward_dim="Overall",
                     use_norm=True, save_fps=8, num_frames=None, fps=None, max_pixels=None, **kw):
    from .videoalign import VideoAlignScorer
    scorer = VideoAlignScorer(device=device, load_from_pretrained=load_from_pretrained,
                              load_from_pretrained_step=load_from_pretrained_step, reward_dim=reward_dim,
                              use_norm=use_norm, num_frames=num_frames, fps=fps, max_pixels=max_pixels,
                              save_fps=save_fps)

    def _fn(images, prompts, metadata):
        if isinstance(images, torch.Tensor):
            if images.dim() == 5 and images.shape[1] == 3:           # [B, C, T, H, W] → [B, T, H, W, C]
                images = images.permute(0, 2, 3, 4, 1)
            if images.dtype != torch.uint8:
                x = images.float()
                if x.min() < 0:                                       # VAE output in [-1, 1]
                    x = (x + 1) * 0.5
                images = (x * 255).round().clamp(0, 255).to(torch.uint8)
            images = [v.cpu() for v in images]
        return scorer(images, prompts), {}
    return _fn


SCORES = {"videoalign": videoalign_score, "latent_mlp": latent_mlp_score}


def multi_score(device, score_dict: Dict[str, float], **score_kwargs):
    fns = {}
    for name, w in score_dict.items():
        if name not in SCORES:
            raise ValueError(f"[multi_score] unsupported score '{name}'; available: {list(SCORES)}")
        fns[name] = SCORES[name](device, **score_kwargs.get(name, {}))

    def _fn(images, prompts, metadata, ref_images=None, only_strict=True):
        details, total = {}, None
        for name, w in score_dict.items():
            s, _ = fns[name](images, prompts, metadata)
            details[name] = s
            ws = np.asarray(s, dtype=np.float64) * w
            total = ws if total is None else total + ws
        details["avg"] = total.tolist()
        return details, {}
    return _fn
