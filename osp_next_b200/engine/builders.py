"""Construction of models, schedulers, encoders and process meshes from a config dict.

Shared by ``train/train_osp.py``, ``train/train_osp_RL.py`` and
``infer/infer_osp.py`` (reference drivers: train_osp.py:121-266,
train_osp_RL.py:700-879, infer_osp.py:82-200).
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.distributed as dist

from ..models import models, models_blocks_to_float, models_main_block
from ..parallel.checkpoint import Checkpointer, load_full_state_dict
from ..parallel.sp import SPRuntime, attach_sp, build_sp_groups
from ..schedulers import schedulers
from ..utils.utils import to_dtype


def world() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def device() -> torch.device:
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def build_fsdp_mesh(config):
    """(ddp, fsdp) mesh (HSDP when ddp > 1), reference train_osp.py:121-130."""
    from torch.distributed.device_mesh import init_device_mesh
    W = world()
    fsdp = min(config.get("fsdp_size", W), W)
    ddp = config.get("ddp_size", W // fsdp)
    if ddp * fsdp != W:
        raise ValueError(f"ddp_size·fsdp_size = {ddp}·{fsdp} != world {W}")
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if ddp > 1:
        return init_device_mesh(dev, (ddp, fsdp), mesh_dim_names=("ddp", "fsdp"))
    return init_device_mesh(dev, (fsdp,), mesh_dim_names=("fsdp",))


def build_sp(config, num_heads: int) -> SPRuntime:
    """SSP × Ulysses (× CFG) groups; the data-parallel degree is what remains."""
    ssp = config.get("skiparse_sp_size", 1) if config.get("use_skiparse_sequence_parallel", False) else 1
    ul = config.get("sp_size", 1) if config.get("use_sequence_parallel", False) else 1
    cfg = config.get("cfg_parallel_size", 1)
    if ssp * ul * cfg == 1 or world() == 1:
        return SPRuntime(__import__("osp_next_b200.models.layout", fromlist=["ParallelSpec"]).ParallelSpec())
    return build_sp_groups(num_heads, skiparse_sp_size=ssp, sp_size=ul, cfg_size=cfg)


def latent_grid(model, data_cfg, vae_stride=(4, 8, 8)):
    """Patch grid (T, H, W) of the data config's samples: Wan VAE strides, then the
    model's patch size."""
    dc = data_cfg.get("dataset_config", {})
    f, h, w = dc.get("sample_num_frames", 81), dc.get("sample_height", 480), dc.get("sample_width", 832)
    pt, ph, pw = model.patch_size
    return (((f - 1) // vae_stride[0] + 1) // pt, h // vae_stride[1] // ph, w // vae_stride[2] // pw)


def build_model(config, dev=None, dtype=torch.float32):
    name = config.get("model_name", "osp_next")
    mcfg = dict(config.get("model_config", {}))
    ckpt = mcfg.pop("pretrained_model_dir_or_checkpoint", None)
    dev = dev or device()
    with torch.device(dev):
        model = models[name](**mcfg)
    model = model.to(dtype)
    if ckpt and os.path.exists(ckpt):
        path = ckpt
        if os.path.isdir(ckpt):
            cands = [f for f in os.listdir(ckpt) if f.endswith((".safetensors", ".pt", ".pth"))]
            if not cands:
                raise FileNotFoundError(f"no weights in {ckpt}")
            path = os.path.join(ckpt, sorted(cands)[0])
        Checkpointer().load_state_dict(model, load_full_state_dict(path))
    return model


def build_scheduler(config):
    sc = dict(config.get("scheduler_config", {}))
    name = sc.pop("scheduler_name", "flow_matching")
    return schedulers[name](**sc)


def build_vae(config, dev=None):
    vc = config.get("vae_config", {})
    from ..models.vae import WanVAE
    return WanVAE(vae_pth=vc.get("vae_path"), dtype=to_dtype(vc.get("dtype", "fp32")), device=dev or device())


def build_text_encoder(config, dev=None, mesh=None):
    """umT5 encoder; with ``text_encoder_config.use_fsdp`` it is FSDP2-sharded over ``mesh``
    (default: 8-way shards replicated over the rest of the world, as the reference)."""
    tc = config.get("text_encoder_config", {})
    from ..models.t5 import T5EncoderModel, t5_mesh
    use_fsdp = bool(tc.get("use_fsdp", False)) and dist.is_initialized() and world() > 1
    if use_fsdp and mesh is None:
        mesh = t5_mesh(world(), tc.get("fsdp_shard_size", 8), "cuda" if torch.cuda.is_available() else "cpu")
    return T5EncoderModel(text_len=tc.get("text_len", 512), dtype=to_dtype(tc.get("dtype", "bf16")),
                          device=dev or device(), checkpoint_path=tc.get("checkpoint_path"),
                          tokenizer_path=tc.get("text_tokenizer_path"), use_fsdp=use_fsdp, device_mesh=mesh)


def fsdp_wrap(model, config, mesh, weight_dtype=torch.bfloat16):
    from ..parallel.fsdp import FSDP2_mix_wrapper, set_modules_to_forward_prefetch
    name = config.get("model_name", "osp_next")
    FSDP2_mix_wrapper(model, mesh, weight_dtype, main_block_to_half=models_main_block[name],
                      blocks_to_float=models_blocks_to_float[name],
                      reshard_after_forward=config.get("reshard_after_forward", None),
                      cpu_offload=config.get("model_cpu_offload", False))
    n = config.get("explicit_prefetching_num_blocks", 0)
    if n:
        set_modules_to_forward_prefetch(list(model.blocks), n)
    return model
