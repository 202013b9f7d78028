"""Dump a Wan-2.1 diffusers directory to one state-dict file (reference: merge_wan_weights.py).

python merge_wan_weights.py --src Wan2.1-T2V-14B --out Wan2.1-T2V-14B/want2v_14b.pt
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from osp_next_b200.models.pretrained import load_pretrained_state_dict  # noqa: E402

if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    torch.save(load_pretrained_state_dict(a.src), a.out)
