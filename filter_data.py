"""Filter an annotation file with WanVideoFilter and write the metadata store
(reference: filter_data.py; LMDB when available, JSONL otherwise).

python filter_data.py --filter_config configs/filter_config.yaml
"""
import os
import sys
from argparse import ArgumentParser

import yaml

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from osp_next_b200.data.utils.meta_store import JSONLMetaWriter, open_meta_reader  # noqa: E402
from osp_next_b200.data.utils.wan_utils import WanVideoFilter  # noqa: E402

if __name__ == "__main__":
    ap = ArgumentParser()
    ap.add_argument("--filter_config", default="configs/filter_config.yaml")
    a = ap.parse_args()
    cfg = yaml.safe_load(open(a.filter_config, encoding="utf-8"))
    flt = WanVideoFilter(**cfg)
    samples = flt.filter_data_samples_force_shape()
    print(flt.stats)
    out = cfg["save_path"]
    if out.endswith(".jsonl"):
        w = JSONLMetaWriter(out)
    else:
        from osp_next_b200.data.utils.meta_store import LMDBWriter
        w = LMDBWriter(out)
    w.write(samples)
    w.close()
    r = open_meta_reader(out)
    print(len(r), r.getitem(0) if len(r) else None)
