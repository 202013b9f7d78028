"""Convert a raw state dict (.pt / .safetensors) into a diffusers-layout model directory
(reference: convert_to_diffusers_weights.py).

python convert_to_diffusers_weights.py --weights model_state_dict.pt --config configs/infer/osp_14b.yaml --out <dir>
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from osp_next_b200.models import models  # noqa: E402
from osp_next_b200.parallel.checkpoint import load_full_state_dict  # noqa: E402
from osp_next_b200.utils.config import load_config  # noqa: E402

if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--weights", required=True)
    ap.add_argument("--config", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    cfg = load_config(a.config)
    mc = dict(cfg["model_config"])
    mc.pop("pretrained_model_dir_or_checkpoint", None)
    model = models[cfg.get("model_name", "osp_next")](**mc)
    missing, unexpected = model.load_state_dict(load_full_state_dict(a.weights), strict=False)
    print(f"missing_keys: {missing}\nunexpected_keys: {unexpected}")
    model.save_pretrained(a.out)
