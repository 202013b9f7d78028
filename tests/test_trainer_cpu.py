"""SFT trainer on CPU (tiny model, synthetic latents): the profiling window writes a
chrome trace per traced iteration and stops the run, metrics go to JSONL, and a second
run resumes from the saved checkpoint."""
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(out, **kw):
    cfg = {
        "model_name": "osp_next", "seed": 0, "output_dir": out, "training_iteration": 100, "max_steps": 3,
        "fsdp_size": 1, "gradient_checkpointing": False, "log_interval": 1, "save_interval": 2,
        "weight_dtype": "fp32", "ema_decay": 0.99, "metrics_file": os.path.join(out, "metrics.jsonl"),
        "model_config": dict(dim=64, ffn_dim=128, num_heads=2, num_layers=2, text_len=8,
                             skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=0),
        "scheduler_config": {"scheduler_name": "flow_matching", "use_logitnorm_time_sampling": True},
        "data_config": {"batch_size": 1, "num_workers": 0, "pin_memory": False, "dataset_name": "t2v_random_latent",
                        "dataset_config": {"sample_height": 64, "sample_width": 64, "sample_num_frames": 5,
                                           "text_max_length": 8}},
        "optimizer_config": {"lr": 1e-4, "weight_decay": 0.0},
        "timeout_s": 120,
    }
    cfg.update(kw)
    return cfg


def _main():
    sys.path.insert(0, os.path.join(ROOT, "train"))
    import train_osp
    return train_osp.main


def test_profiling_window_traces_and_stops(tmp_path, monkeypatch):
    for k, v in dict(MASTER_ADDR="127.0.0.1", MASTER_PORT="29631", RANK="0", WORLD_SIZE="1", LOCAL_RANK="0").items():
        monkeypatch.setenv(k, v)
    main = _main()
    out = str(tmp_path)
    times = main(_cfg(out, max_steps=10, profiling={"start": 1, "steps": 1, "exit_after": True}))
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()
    assert os.path.exists(os.path.join(out, "trace_rank0_000000001.json"))
    recs = [json.loads(l) for l in open(os.path.join(out, "metrics.jsonl"))]
    assert [r["iter"] for r in recs] == [1, 2]          # stopped right after the window
    assert all("loss" in r and "clipper/max_grad_norm" in r for r in recs)
    # resume: the checkpoint of iteration 2 is picked up and training continues from there
    main(_cfg(out, max_steps=1))
    if dist.is_initialized():
        dist.destroy_process_group()
    recs = [json.loads(l) for l in open(os.path.join(out, "metrics.jsonl"))]
    assert recs[-1]["iter"] == 3
