"""``save_pretrained`` / ``from_pretrained`` in the diffusers directory layout.

The reference's models are diffusers ``ModelMixin``s (osp_next.py:1025, want2v.py:291);
their checkpoints are a directory with ``config.json`` and
``diffusion_pytorch_model.safetensors`` (or a sharded index).  These helpers
read and write that layout without depending on diffusers.
"""
from __future__ import annotations

import json
import os

import torch

WEIGHTS = "diffusion_pytorch_model.safetensors"
INDEX = "diffusion_pytorch_model.safetensors.index.json"


def save_pretrained(model, path: str, max_shard_bytes: int = 10 * 1024 ** 3):
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    cfg = dict(getattr(model, "config", {}))
    cfg["_class_name"] = type(model).__name__
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    sd = {k: v.detach().contiguous().cpu() for k, v in model.state_dict().items()}
    total = sum(v.numel() * v.element_size() for v in sd.values())
    if total <= max_shard_bytes:
        save_file(sd, os.path.join(path, WEIGHTS))
        return
    shards, cur, size = [], {}, 0
    for k, v in sd.items():
        b = v.numel() * v.element_size()
        if cur and size + b > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = v
        size += b
    shards.append(cur)
    wmap = {}
    for i, sh in enumerate(shards):
        name = f"diffusion_pytorch_model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, name))
        wmap.update({k: name for k in sh})
    with open(os.path.join(path, INDEX), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": wmap}, f, indent=2)


def load_pretrained_state_dict(path: str) -> dict:
    from safetensors.torch import load_file
    if os.path.exists(os.path.join(path, WEIGHTS)):
        return load_file(os.path.join(path, WEIGHTS))
    with open(os.path.join(path, INDEX)) as f:
        files = sorted(set(json.load(f)["weight_map"].values()))
    sd = {}
    for fn in files:
        sd.update(load_file(os.path.join(path, fn)))
    return sd


def from_pretrained(cls, path: str, device="cpu", dtype=None, **overrides):
    with open(os.path.join(path, "config.json")) as f:
        cfg = json.load(f)
    cfg = {k: v for k, v in cfg.items() if not k.startswith("_")}
    cfg.update(overrides)
    with torch.device(device):
        model = cls(**cfg)
    sd = load_pretrained_state_dict(path)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    if missing or unexpected:
        print(f"from_pretrained: missing {len(missing)} unexpected {len(unexpected)} keys")
    return model.to(dtype) if dtype is not None else model
