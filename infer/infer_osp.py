"""T2V inference driver (reference: infer/infer_osp.py:38-275).

``torchrun --nproc-per-node N infer/infer_osp.py --config configs/infer/osp_14b.yaml``

Builds the VAE, tokenizer + T5, scheduler and DiT from the YAML, sets up the SP
layout (SSP × Ulysses, plus optional CFG-parallel), then walks the prompt file:
each data-parallel replica takes every ``dp``-th prompt, runs the T2V pipeline
and the first rank of each SP group writes the mp4; finally the videos are
gathered to rank 0 and tiled into a grid.  Weights are replicated per GPU (the
14B bf16 DiT is 28.6 GB, well within one B200) instead of being FSDP-sharded as
in the reference, which removes a full weight all-gather per forward.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from osp_next_b200 import ops  # noqa: E402
from osp_next_b200.engine import builders as B  # noqa: E402
from osp_next_b200.parallel.cfg import CFGParallel  # noqa: E402
from osp_next_b200.parallel.dist_utils import gather_tensor_list_to_one, setup_distributed_env  # noqa: E402
from osp_next_b200.parallel.sp import attach_sp  # noqa: E402
from osp_next_b200.parallel.sp_state import sp_state  # noqa: E402
from osp_next_b200.pipelines import pipelines  # noqa: E402
from osp_next_b200.utils.config import load_config  # noqa: E402
from osp_next_b200.utils.log_utils import get_logger, log_on_main_process  # noqa: E402
from osp_next_b200.utils.random_utils import set_seed  # noqa: E402
from osp_next_b200.utils.utils import to_dtype  # noqa: E402


def read_prompts(path):
    with open(path, encoding="utf-8") as f:
        return [l.strip() for l in f if l.strip()]


def main(config):
    logger = get_logger()
    setup_distributed_env(timeout_s=config.get("timeout_s", 600))
    rank, W = B.rank(), B.world()
    dev = B.device()
    set_seed(config.get("seed", 42))
    wdt = to_dtype(config.get("weight_dtype", "bf16"))
    mcfg = config.get("model_config", {})
    sp_rt = B.build_sp(config, mcfg.get("num_heads", 16))
    cfg_size = config.get("cfg_parallel_size", 1)
    gsp = sp_rt.spec.world * cfg_size
    dp = max(1, W // gsp)
    dp_rank = rank // gsp

    model = B.build_model(config, dev, torch.float32).to(wdt).eval()
    for n, p in model.named_parameters():
        if "norm" in n or "modulation" in n:
            p.data = p.data.float()
    attach_sp(model, sp_rt)
    model.enable_text_kv_cache(True)
    scheduler = B.build_scheduler(config)
    vae = B.build_vae(config, dev)
    t5 = B.build_text_encoder(config, dev)
    pipe = pipelines[config.get("pipeline_name", "t2v")](vae=vae, tokenizer=t5.tokenizer, text_encoder=t5,
                                                         predictor=model, scheduler=scheduler)
    cfg_par = CFGParallel(sp_state.cfg_group) if cfg_size > 1 else None
    prompts = read_prompts(config["prompt_txt"])
    out_dir = config.get("output_dir", "./output")
    os.makedirs(out_dir, exist_ok=True)
    bs = config.get("batch_size", 1)
    videos = []
    from osp_next_b200.data.utils.video_io import save_video, video_grid
    for i in range(dp_rank * bs, len(prompts), dp * bs):
        batch = prompts[i:i + bs]
        vid = pipe(batch, num_frames=config.get("num_frames", 49), height=config.get("height", 480),
                   width=config.get("width", 832), seed=config.get("seed", 42) + i, device=dev,
                   cfg_parallel=cfg_par)
        ops.check_device_errors(dev, where=f"prompt {i}")    # VAE decode / final step of this video
        if rank % gsp == 0:
            for j, v in enumerate(vid):
                save_video(v, os.path.join(out_dir, f"{i + j:05d}.mp4"), fps=config.get("save_fps", 16))
                videos.append(v)
        log_on_main_process(logger, f"prompt {i} done")
    if W > 1:
        gathered = gather_tensor_list_to_one(videos, dst=0)
        if rank == 0 and gathered:
            save_video(video_grid(gathered), os.path.join(out_dir, "grid.mp4"), fps=config.get("save_fps", 16))
    elif videos:
        save_video(video_grid(videos), os.path.join(out_dir, "grid.mp4"), fps=config.get("save_fps", 16))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    a = ap.parse_args()
    main(load_config(a.config))
    if dist.is_initialized():
        dist.destroy_process_group()
