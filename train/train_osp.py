"""Flow-matching SFT of the OSP-Next DiT (reference: train/train_osp.py:52-561).

``torchrun --nproc-per-node N train/train_osp.py --config configs/train/osp_14b.yaml``

Steps per iteration, as in the reference: fetch a batch (every ``global_sp``
steps, then share it inside the SP group with the encoder cache), VAE + T5
encode (or take synthetic latents / embeddings with ``dataset_name:
t2v_random_latent``), ``q_sample`` with logit-normal σ and resolution-dependent
shift, broadcast ``x_t, noise, σ`` inside the SP group, forward (FSDP2 mixed
precision; GEMMs and attention on the sm_100a kernels), velocity MSE, backward,
adaptive clipping + fused AdamW + EMA on the accumulation boundary, logging
(loss averaged over ranks, lr, grad norm, tokens/s from device timers, max over
ranks), atomic checkpoints in the reference layout with resume from the newest.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from osp_next_b200 import ops  # noqa: E402
from osp_next_b200.data import ospnext_collators, ospnext_datasets, ospnext_samplers  # noqa: E402
from osp_next_b200.engine import builders as B  # noqa: E402
from osp_next_b200.parallel.checkpoint import Checkpointer  # noqa: E402
from osp_next_b200.parallel.dist_utils import gather_data_from_all_ranks, setup_distributed_env  # noqa: E402
from osp_next_b200.parallel.ema import FSDPEMAModel  # noqa: E402
from osp_next_b200.parallel.optim import FusedAdamW  # noqa: E402
from osp_next_b200.parallel.sp import attach_sp  # noqa: E402
from osp_next_b200.parallel.sp_state import sp_state  # noqa: E402
from osp_next_b200.utils.clip_grads import AdaptiveGradClipper  # noqa: E402
from osp_next_b200.utils.config import load_config  # noqa: E402
from osp_next_b200.utils.constant import PROMPT_IDS, PROMPT_MASK, VIDEO  # noqa: E402
from osp_next_b200.utils.encoder_cache import EncoderCacheManager  # noqa: E402
from osp_next_b200.utils.log_utils import MetricsLogger, get_logger, log_on_main_process  # noqa: E402
from osp_next_b200.utils.profiling import ProfileWindow, enable_nvtx, nvtx_range  # noqa: E402
from osp_next_b200.utils.random_utils import set_deterministic, set_seed  # noqa: E402
from osp_next_b200.utils.utils import to_dtype  # noqa: E402


def _sp_broadcast(tensors, group):
    if group is None or dist.get_world_size(group) == 1:
        return tensors
    src = dist.get_global_rank(group, 0)
    for t in tensors:
        dist.broadcast(t, src=src, group=group)
    return tensors


def main(config, on_step=None):
    """Train per ``config``.  ``on_step(it, step_ms, tokens_per_step)`` (optional) is called on
    every rank after each optimizer step, once the step's device work has finished.
    Returns the per-step device times (ms, CUDA events on this rank)."""
    logger = get_logger()
    setup_distributed_env(timeout_s=config.get("timeout_s", 600))
    rank, W = B.rank(), B.world()
    dev = B.device()
    seed = config.get("seed", 42)
    if config.get("deterministic_training", False):
        set_deterministic(True)
    weight_dtype = to_dtype(config.get("weight_dtype", "bf16"))
    mcfg = config.get("model_config", {})
    data_cfg = config.get("data_config", {})
    opt_cfg = config.get("optimizer_config", {})
    output_dir = config.get("output_dir", "./output")
    iters = config.get("training_iteration", 1000000)
    max_steps = config.get("max_steps", None)
    accum = config.get("gradient_accumulation_steps", 1)
    log_interval = config.get("log_interval", 1)
    save_interval = config.get("save_interval", 1000)

    # ------------------------------------------------------------ parallel layout
    sp_rt = B.build_sp(config, mcfg.get("num_heads", 16))
    gsp = sp_rt.spec.world
    set_seed(seed + rank // max(1, gsp))           # ranks of one SP group draw the same noise
    mesh = B.build_fsdp_mesh(config) if (W > 1 and dist.is_initialized()) else None

    # ------------------------------------------------------------ model / optimizer
    model = B.build_model(config, dev, torch.float32)
    attach_sp(model, sp_rt)
    if config.get("gradient_checkpointing", False):
        model.set_gradient_checkpointing(True)
    if mesh is not None:
        B.fsdp_wrap(model, config, mesh, weight_dtype)
    p2p_arenas = None
    if mesh is not None and dev.type == "cuda" and config.get("fsdp_p2p_collectives", True):
        # block parameter all-gather / gradient reduce-scatter over NVLink peer memory
        from osp_next_b200.parallel.fsdp_comm import enable_p2p_fsdp
        fsdp_dim = mesh["fsdp"] if "ddp" in (mesh.mesh_dim_names or ()) else mesh
        p2p_arenas = enable_p2p_fsdp(list(model.blocks), fsdp_dim.get_group(), device=dev,
                                     barrier_limit_s=config.get("fsdp_p2p_timeout_s", 60.0))
    sp_p2p = None
    if gsp > 1 and dev.type == "cuda" and config.get("ssp_p2p_exchange", True):
        # SSP layout changes and Ulysses all-to-alls (forward and backward) over NVLink
        from osp_next_b200.parallel.sp import enable_p2p_exchange
        sp_p2p = enable_p2p_exchange(model, data_cfg.get("batch_size", 1), B.latent_grid(model, data_cfg), dev,
                                     limit_s=config.get("ssp_p2p_timeout_s", 60.0))
    ema = FSDPEMAModel(model, config.get("ema_decay", 0.9999), config.get("ema_update_interval", 1)) \
        if config.get("ema_decay", 0) else None
    opt = FusedAdamW([p for p in model.parameters() if p.requires_grad], lr=opt_cfg.get("lr", 1e-5),
                     betas=tuple(opt_cfg.get("betas", (0.9, 0.999))), eps=opt_cfg.get("eps", 1e-15),
                     weight_decay=opt_cfg.get("weight_decay", 0.0))
    shard_group = None
    if mesh is not None:
        shard_group = (mesh["fsdp"] if "ddp" in (mesh.mesh_dim_names or ()) else mesh).get_group()
    clipper = AdaptiveGradClipper(init_max_grad_norm=config.get("init_max_grad_norm", 1.0),
                                  model_parallel_group=shard_group,
                                  legacy_group_sum=config.get("legacy_clip_group_sum", False))
    ckpt = Checkpointer(output_dir)
    start_it = ckpt.last_training_iteration
    if start_it > 0:
        ckpt.load_model(model)
        ckpt.load_optim(model, opt)
        if ema is not None:
            ema.store(model)
            ckpt.load_model(model, ema=True)
            ema.model_copy_to_ema(model)
            ema.restore(model)
        clipper.load(ckpt.iter_dir(start_it))
        ckpt.load_rng()
        if opt_cfg.get("resume_override_lr", False):
            for g in opt.param_groups:
                g["lr"] = opt_cfg.get("resume_lr", g["lr"])
        log_on_main_process(logger, f"resumed from iteration {start_it}")

    # ------------------------------------------------------------ data
    scheduler = B.build_scheduler(config)
    ds_name = data_cfg.get("dataset_name", "t2v_random")
    ds = ospnext_datasets[ds_name](**data_cfg.get("dataset_config", {}))
    latent_mode = ds_name == "t2v_random_latent"
    sampler = ospnext_samplers[data_cfg.get("sampler_name", "stateful_distributed")](
        ds, num_replicas=W, rank=rank, shuffle=data_cfg.get("shuffle", True), seed=seed,
        drop_last=data_cfg.get("drop_last", True))
    collate = ospnext_collators["latent" if latent_mode else data_cfg.get("collator_name", "wan_t2v")]()
    loader = torch.utils.data.DataLoader(ds, batch_size=data_cfg.get("batch_size", 1), sampler=sampler,
                                         num_workers=data_cfg.get("num_workers", 0), collate_fn=collate,
                                         pin_memory=data_cfg.get("pin_memory", True), drop_last=True)
    ckpt.load_dataloader(sampler)
    vae = t5 = None
    if not latent_mode:
        vae = B.build_vae(config, dev)
        t5 = B.build_text_encoder(config, dev)
    cache = EncoderCacheManager(sp_rt.global_sp_group if gsp > 1 else None)
    it_data = iter(loader)

    metrics_file = config.get("metrics_file")
    wb = config.get("wandb_config", {}) or {}
    metrics = MetricsLogger(metrics_file, use_wandb=wb.get("project_name") is not None,
                            project=wb.get("project_name") or "osp_next_b200", run_name=wb.get("exp_name"),
                            config=config)
    profile = ProfileWindow(config.get("profiling", False), output_dir, rank)
    if config.get("nvtx", False):
        enable_nvtx(True)
    step_times, tokens_per_step = [], None
    model.train()
    it = start_it
    while it < iters and (max_steps is None or it - start_it < max_steps):
        if dev.type == "cuda":
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        with profile(it):
            for micro in range(accum):
                with nvtx_range("data"):
                    if cache.need_encode():
                        batch = next(it_data)
                        with torch.no_grad():
                            if latent_mode:
                                lat = batch["latents"].to(dev, non_blocking=True)
                                txt = batch["text"].to(dev, non_blocking=True).to(weight_dtype)
                            else:
                                lat = vae.encode(batch[VIDEO].to(dev))
                                txt = t5(batch[PROMPT_IDS].to(dev), batch[PROMPT_MASK].to(dev)).to(weight_dtype)
                        cache.set_cache([lat.float(), txt])
                    lat, txt = cache()
                    q = scheduler.q_sample(lat)
                    x_t, noise, sig, t = q["x_t"], q["prior_dist"], q["sigmas"], q["timesteps"]
                    _sp_broadcast([x_t, noise, sig, t], sp_rt.global_sp_group if gsp > 1 else None)
                tokens_per_step = x_t.shape[0] * (x_t.shape[2] * x_t.shape[3] * x_t.shape[4] // 4) * W // max(1, gsp)
                with nvtx_range("forward"):
                    pred = model(x_t.to(weight_dtype), t, txt)
                    loss = scheduler.training_losses(pred, lat, noise, sigmas=sig)[0] / accum
                with nvtx_range("backward"):
                    loss.backward()
        with nvtx_range("optimizer"):
            params = [p for p in model.parameters() if p.grad is not None]
            opt.grad_scale = clipper.adaptive_clip(params, apply=False)
            opt.step()
            opt.zero_grad(set_to_none=True)
        it += 1
        if ema is not None:
            ema.update(model, it)
        if dev.type == "cuda":
            ev1.record()
            torch.cuda.synchronize()
            ms = ev0.elapsed_time(ev1)
            step_times.append(ms)
            if on_step is not None:
                on_step(it, ms, tokens_per_step)
        # a bounded device wait that gave up (a stalled or dead peer in an NVLink collective)
        # leaves this step's gradients invalid: stop every rank before logging or saving;
        # a restart resumes from the newest checkpoint
        ops.check_device_errors_all_ranks(dev, where=f"training iteration {it}")
        if it % log_interval == 0:
            lv = gather_data_from_all_ranks(loss.detach().float() * accum).mean().item()
            ms_max = step_times[-1] if step_times else 0.0
            if dist.is_initialized() and dev.type == "cuda":
                tt = torch.tensor([ms_max], device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                ms_max = float(tt.item())
            rec = {"iter": it, "loss": lv, "lr": opt.param_groups[0]["lr"],
                   "grad_norm": clipper.grad_norm_before_clip, "max_grad_norm": clipper.max_grad_norm,
                   "step_ms": ms_max,
                   "tokens_per_s": (tokens_per_step / (ms_max / 1000.0)) if ms_max else None}
            log_on_main_process(logger, json.dumps(rec))
            metrics.log(dict(rec, **{f"clipper/{k}": v for k, v in clipper.state_dict().items()
                                     if isinstance(v, (int, float))}), step=it)
        if it % save_interval == 0:
            ckpt.save(it, model, opt, ema, sampler, clipper)
        if profile.finished(it):
            log_on_main_process(logger, f"profiling window done at iteration {it}; traces in {output_dir}")
            break
    if p2p_arenas is not None:
        from osp_next_b200.parallel.fsdp_comm import close
        dist.barrier()
        close(p2p_arenas)
    if sp_p2p is not None:
        sp_p2p.close()
    metrics.close()
    return step_times


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    a = ap.parse_args()
    main(load_config(a.config))
    if dist.is_initialized():
        dist.destroy_process_group()
