"""YAML configs with the reference's keys (reference: §config — drivers read a plain
dict with ``config.get(key, default)``).  ``load_config`` returns that dict and
warns about top-level keys no driver of this framework reads, so typos surface."""
from __future__ import annotations

import logging
import warnings

import yaml

KNOWN_KEYS = {
    "model_name", "task", "seed", "output_dir", "training_iteration", "fsdp_size", "ddp_size", "sp_size",
    "skiparse_sp_size", "cfg_parallel_size", "use_sequence_parallel", "use_skiparse_sequence_parallel",
    "reshard_after_forward", "explicit_prefetching_num_blocks", "gradient_checkpointing",
    "gradient_accumulation_steps", "init_max_grad_norm", "log_interval", "save_interval", "weight_dtype",
    "ema_decay", "ema_update_interval", "save_with_dcp_api", "model_cpu_offload", "encoder_cpu_offload",
    "deterministic_training", "profiling", "wandb_config", "model_config", "scheduler_config", "vae_config",
    "text_encoder_config", "data_config", "optimizer_config", "pipeline_name", "prompt_txt", "batch_size",
    "num_frames", "height", "width", "save_fps", "num_epochs", "resume_epoch", "lora_config", "rl_config",
    "metrics_file", "max_steps", "timeout_s", "legacy_clip_group_sum", "fsdp_p2p_collectives",
}


def load_config(path: str) -> dict:
    with open(path) as f:
        cfg = yaml.safe_load(f) or {}
    unknown = sorted(set(cfg) - KNOWN_KEYS)
    if unknown:
        warnings.warn(f"config keys not used by osp_next_b200: {unknown}")
    return cfg
