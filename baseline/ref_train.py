"""Reference arm of ``bench.py --mode train``: the unmodified reference's training step.

Runs one flow-matching training step per iteration with the reference's own public
pieces, in the order of its trainer (reference train/train_osp.py:300-330 for set-up,
:420-500 for the step): ``OSPNextModel`` built on the meta device, ``FSDP2_mix_wrapper``
over a (ddp, fsdp) mesh, ``reset_parameters``, gradient checkpointing, its FSDP EMA,
``torch.optim.AdamW``, its ``AdaptiveGradClipper``; per step ``q_sample``, broadcast
inside the global SP group, autocast bf16 forward, ``training_losses``, backward, loss
gather, adaptive clip, AdamW, EMA.  Latents and text embeddings are synthetic (as in the
framework arm), so the reference's VAE / T5 encoders and data loader are not run.
"""
from __future__ import annotations

import math
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import ref_harness  # noqa: E402


def train(cfg: dict, on_step) -> None:
    osp, fm = ref_harness.import_reference(disable_compile=False, force_sdpa=not ref_harness.fa2_usable())
    from torch.distributed.device_mesh import init_device_mesh
    from ospnext.distributed.fsdp2_wrapper import FSDP2_mix_wrapper
    from ospnext.distributed.fsdp_ema import FSDPEMAModel
    from ospnext.distributed.sp_state import sp_state
    from ospnext.distributed.utils import gather_data_from_all_ranks
    from ospnext.modules import models, models_main_block, models_blocks_to_float, models_blocks_to_output_float
    from ospnext.schedulers import schedulers
    from ospnext.utils.clip_grads import AdaptiveGradClipper

    world = dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    mcfg = dict(cfg["model_config"])
    fsdp = min(cfg.get("fsdp_size", world), world)
    ddp_fsdp_mesh = init_device_mesh("cuda", (world // fsdp, fsdp), mesh_dim_names=("ddp", "fsdp"))
    ssp = cfg.get("skiparse_sp_size", 1) if cfg.get("use_skiparse_sequence_parallel", False) else 1
    gsp = ssp
    global_sp_group = None
    if gsp > 1:
        mesh = init_device_mesh("cuda", (world // gsp, ssp, 1), mesh_dim_names=("dp", "skiparse_sp", "sp"))
        global_sp_group = mesh["skiparse_sp", "sp"]._flatten().get_group()
        sp_state.reset(global_sp_group=global_sp_group, sp_group=mesh["sp"].get_group(),
                       skiparse_sp_group=mesh["skiparse_sp"].get_group(), full_sp_group=mesh["sp"].get_group())
        if mcfg.get("num_full_blocks", 0) > 0:
            heads = mcfg["num_heads"]
            full = gsp if (gsp <= heads and heads % gsp == 0) else math.gcd(heads, gsp)
            dummy = init_device_mesh("cuda", (world // full, full), mesh_dim_names=("dummy", "full_sp"))
            sp_state.reset(full_sp_group=dummy["full_sp"].get_group())

    torch.manual_seed(cfg.get("seed", 1024))
    with torch.device("meta"):
        model = models["osp_next"](**mcfg)
    model.train()
    FSDP2_mix_wrapper(model, dp_mesh=ddp_fsdp_mesh, weight_dtype=torch.bfloat16,
                      main_block_to_half=models_main_block["osp_next"],
                      blocks_to_float=models_blocks_to_float["osp_next"],
                      blocks_to_output_float=models_blocks_to_output_float["osp_next"],
                      reshard_after_forward=cfg.get("reshard_after_forward", None), cpu_offload=False)
    model.to_empty(device=device)
    model.reset_parameters()
    model.set_gradient_checkpointing(True)
    ema = FSDPEMAModel(model, decay=cfg.get("ema_decay", 0.9999), update_interval=cfg.get("ema_update_interval", 1))
    oc = cfg.get("optimizer_config", {})
    opt = torch.optim.AdamW(model.parameters(), lr=oc.get("lr", 1e-5), betas=tuple(oc.get("betas", (0.9, 0.999))),
                            weight_decay=oc.get("weight_decay", 0.0), eps=oc.get("eps", 1e-15))
    clipper = AdaptiveGradClipper(init_max_grad_norm=cfg.get("init_max_grad_norm", 1.0),
                                  model_parallel_group=ddp_fsdp_mesh["fsdp"].get_group())
    sc = dict(cfg.get("scheduler_config", {}))
    scheduler = schedulers[sc.pop("scheduler_name", "flow_matching")](**sc)

    dc = cfg["data_config"]["dataset_config"]
    T = (dc["sample_num_frames"] - 1) // 4 + 1
    H, W = dc["sample_height"] // 8, dc["sample_width"] // 8
    g = torch.Generator().manual_seed(1234 + dist.get_rank() // gsp)
    lat_h = torch.randn(1, 16, T, H, W, generator=g).pin_memory()
    txt_h = torch.randn(1, mcfg["text_len"], 4096, generator=g).to(torch.bfloat16).pin_memory()
    tokens = T * (H // 2) * (W // 2) * (world // gsp)
    for it in range(1, cfg["max_steps"] + 1):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        latents = lat_h.to(device, non_blocking=True)
        text = txt_h.to(device, non_blocking=True)
        q = scheduler.q_sample(latents)
        x_t = q["x_t"].to(torch.bfloat16)
        prior, sig, ts = q["prior_dist"], q["sigmas"], q["timesteps"]
        if global_sp_group is not None:
            for t in (x_t, prior, sig, ts):
                dist.broadcast(t, group_src=0, group=global_sp_group)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(x_t, ts, text)
        loss = scheduler.training_losses(out, latents, prior)[0]
        loss.backward()
        gather_data_from_all_ranks(loss.detach().unsqueeze(0), dim=0).mean().item()
        clipper.adaptive_clip(model.parameters())
        opt.step()
        opt.zero_grad()
        ema.update(model, it)
        ev1.record()
        torch.cuda.synchronize()
        on_step(it, ev0.elapsed_time(ev1), tokens)
