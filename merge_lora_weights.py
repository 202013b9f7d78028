"""Fold a LoRA adapter into the base DiT and save the merged weights
(reference: merge_lora_weights.py:5-87, which uses PEFT merge_and_unload).

python merge_lora_weights.py --base <diffusers dir | .pt/.safetensors> --lora <lora-checkpoint-N> \
    --out <dir> [--config configs/infer/osp_14b.yaml]
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from osp_next_b200.models.lora import LoraModel  # noqa: E402
from osp_next_b200.models.osp_next import OSPNextModel  # noqa: E402
from osp_next_b200.parallel.checkpoint import load_full_state_dict  # noqa: E402
from osp_next_b200.utils.config import load_config  # noqa: E402


def load_lora_and_merge(model, lora_dir, lora_rank=None, lora_alpha=None, lora_target_modules=None):
    import json
    cfg_path = os.path.join(lora_dir, "adapter_config.json")
    cfg = json.load(open(cfg_path)) if os.path.exists(cfg_path) else {}
    r = lora_rank or cfg.get("r", 32)
    a = lora_alpha or cfg.get("lora_alpha", 64)
    targets = lora_target_modules or cfg.get("target_modules") or [
        "self_attn.q", "self_attn.k", "self_attn.v", "self_attn.o",
        "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.o"]
    wrapped = LoraModel(model, r=r, lora_alpha=a, target_modules=targets)
    missing = wrapped.load_adapter(lora_dir, strict=True)
    if missing:
        raise RuntimeError(f"LoRA load missing keys, e.g. {missing[:5]}")
    return wrapped.merge_and_unload()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--base", required=True)
    ap.add_argument("--lora", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--config", default=None)
    a = ap.parse_args()
    if os.path.isdir(a.base):
        model = OSPNextModel.from_pretrained(a.base)
    else:
        mc = load_config(a.config)["model_config"] if a.config else {}
        mc.pop("pretrained_model_dir_or_checkpoint", None)
        model = OSPNextModel(**mc)
        model.load_state_dict(load_full_state_dict(a.base), strict=False)
    merged = load_lora_and_merge(model, a.lora)
    merged.save_pretrained(a.out)
    print(f"merged model saved to {a.out}")
