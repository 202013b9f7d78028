"""Mix-GRPO + LoRA reinforcement learning of the OSP-Next DiT (reference: train/train_osp_RL.py:612-1725).

``torchrun --nproc-per-node N train/train_osp_RL.py --config configs/train/osp_14b_RL.yaml``

Per epoch, as in the reference:
  rollout   prompts drawn so each appears ``num_image_per_prompt`` times across the
            world (DistributedKRepeatSampler); CFG sampling with SDE steps for
            ``i < sde_steps`` (log-probs and latents stored) and ODE steps after;
            optional KL reward against the adapter-disabled model;
  reward    ``multi_score`` (VideoAlign on decoded video, or the latent MLP
            scorer), gathered over data-parallel ranks;
  advantage per-prompt mean/std (PerPromptStatTracker), clipped;
  update    for every sample and every trained SDE step: log-prob under the
            current policy (grad through the cond pass, CFG via lerp), PPO-clip
            loss (+β·KL), backward; clip + fused AdamW over LoRA params, LoRA-only
            EMA;
  save      LoRA (+EMA) ``lora-checkpoint-{step}/adapter_model.bin`` with PEFT key
            names, clipper state and ``rl_training_state.json``.
Prompts may also be random text embeddings (``rl_config.synthetic_prompts``), the
BASELINE configuration.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from osp_next_b200.engine import builders as B  # noqa: E402
from osp_next_b200.models.lora import LoraModel  # noqa: E402
from osp_next_b200.parallel.dist_utils import setup_distributed_env  # noqa: E402
from osp_next_b200.parallel.ema import FSDPEMAModel  # noqa: E402
from osp_next_b200.parallel.optim import FusedAdamW  # noqa: E402
from osp_next_b200.parallel.sp import attach_sp  # noqa: E402
from osp_next_b200.rewards import multi_score  # noqa: E402
from osp_next_b200.rl.grpo import (PerPromptStatTracker, compute_log_prob_for_training, grpo_loss,  # noqa: E402
                                   osp_sample_with_logprob, shifted_sigmas)
from osp_next_b200.utils.clip_grads import AdaptiveGradClipper  # noqa: E402
from osp_next_b200.utils.config import load_config  # noqa: E402
from osp_next_b200.utils.log_utils import get_logger, log_on_main_process  # noqa: E402
from osp_next_b200.utils.random_utils import set_seed  # noqa: E402
from osp_next_b200.utils.utils import to_dtype  # noqa: E402

LORA_PREFIX = "lora-checkpoint-"
RL_STATE = "rl_training_state.json"


def save_lora(model: LoraModel, out_dir, step, suffix="", ema=None):
    path = os.path.join(out_dir, f"{LORA_PREFIX}{step}{suffix}")
    if ema is not None:
        ema.store(model)
        ema.ema_copy_to_model(model)
    if B.rank() == 0:
        model.save_pretrained(path)
    if ema is not None:
        ema.restore(model)
    return path


def main(config):
    logger = get_logger()
    setup_distributed_env(timeout_s=config.get("timeout_s", 600))
    rank, W = B.rank(), B.world()
    dev = B.device()
    wdt = to_dtype(config.get("weight_dtype", "bf16"))
    seed = config.get("seed", 42)
    rl = config.get("rl_config", {})
    lc = config.get("lora_config", {})
    mcfg = config.get("model_config", {})
    out_dir = config.get("output_dir", "./output_rl_lora")
    os.makedirs(out_dir, exist_ok=True)

    sp_rt = B.build_sp(config, mcfg.get("num_heads", 16))
    gsp = sp_rt.spec.world
    dp, dp_rank = max(1, W // gsp), rank // max(1, gsp)
    set_seed(seed + dp_rank)
    sp_group = sp_rt.global_sp_group if gsp > 1 else None

    # ------------------------------------------------------------ model + LoRA
    model = B.build_model(config, dev, torch.float32).to(wdt)
    for n, p in model.named_parameters():
        if "norm" in n or "modulation" in n:
            p.data = p.data.float()
    if config.get("gradient_checkpointing", False):
        model.set_gradient_checkpointing(True)
    attach_sp(model, sp_rt)
    targets = lc.get("target_modules", ["self_attn.q", "self_attn.k", "self_attn.v", "self_attn.o"])
    policy = LoraModel(model, r=lc.get("rank", 32), lora_alpha=lc.get("alpha", 64), target_modules=targets)
    for m in policy.lora_modules():
        m.lora_A["default"].to(torch.float32)
        m.lora_B["default"].to(torch.float32)
    if lc.get("lora_path"):
        policy.load_adapter(lc["lora_path"])
    lora_params = [p for n, p in policy.named_parameters() if "lora_" in n]
    for p in lora_params:
        p.data = p.data.float()
    ema = FSDPEMAModel(policy, config.get("ema_decay", 0.9999), config.get("ema_update_interval", 1), lora_only=True) \
        if config.get("ema_decay", 0) else None
    oc = config.get("optimizer_config", {})
    opt = FusedAdamW(lora_params, lr=oc.get("lr", 1e-5), betas=tuple(oc.get("betas", (0.9, 0.999))),
                     eps=oc.get("eps", 1e-8), weight_decay=oc.get("weight_decay", 1e-4))
    clipper = AdaptiveGradClipper(init_max_grad_norm=config.get("init_max_grad_norm", 1.0))
    start_epoch, global_step = 0, 0
    if lc.get("lora_path") and os.path.exists(os.path.join(lc["lora_path"], RL_STATE)):
        with open(os.path.join(lc["lora_path"], RL_STATE)) as f:
            st = json.load(f)
        start_epoch, global_step = st["next_epoch"], st["global_step"]
        clipper.load(lc["lora_path"])

    # ------------------------------------------------------------ rollout setup
    scheduler = B.build_scheduler(config)
    n_steps = rl.get("num_inference_steps", 16)
    sde_steps = rl.get("sde_steps", n_steps)
    g = rl.get("guidance_scale", 5.0)
    k = rl.get("num_image_per_prompt", 4)
    sbs = rl.get("sample_batch_size", 1)
    H, Wd, F = rl.get("height", 480), rl.get("width", 832), rl.get("num_frames", 33)
    lat_shape = (sbs, 16, (F - 1) // 4 + 1, H // 8, Wd // 8)
    text_len = mcfg.get("text_len", 512)
    synthetic = rl.get("synthetic_prompts", rl.get("prompt_file") is None)
    reward_cfg = rl.get("reward_fn", {"latent_mlp": 1.0})
    reward_fn = multi_score(dev, reward_cfg)
    decode = "videoalign" in reward_cfg
    vae = B.build_vae(config, dev) if decode else None
    t5 = None if synthetic else B.build_text_encoder(config, dev)
    prompts = None
    if not synthetic:
        with open(rl["prompt_file"], encoding="utf-8") as fh:
            prompts = [l.strip() for l in fh if l.strip()]
    n_prompt_pool = rl.get("num_prompts", 64)
    neg = torch.zeros(1, text_len, 4096, dtype=wdt, device=dev)
    sigmas = shifted_sigmas(n_steps, getattr(scheduler, "shift", 1.0), dev)
    tracker = PerPromptStatTracker(rl.get("global_std", False))
    train_steps = max(1, int(sde_steps * rl.get("timestep_fraction", 1.0)))

    def embed(pid):
        if synthetic:
            gen = torch.Generator().manual_seed(10_000 + pid)
            return torch.randn(1, text_len, 4096, generator=gen).to(dev, wdt)
        return t5([prompts[pid]]).to(wdt)

    epochs = config.get("num_epochs", 1000)
    import time as _time
    for epoch in range(start_epoch, epochs):
        if dev.type == "cuda":
            torch.cuda.synchronize()
        t_epoch = _time.perf_counter()
        # ------------------------------------------------ rollout
        gen = torch.Generator().manual_seed(seed + epoch)
        m = max(1, (dp * sbs * rl.get("num_batches_per_epoch", 1)) // k)
        pool = torch.randperm(n_prompt_pool if synthetic else len(prompts), generator=gen)[:m].tolist()
        rep = [p for p in pool for _ in range(k)]
        order = torch.randperm(len(rep), generator=gen).tolist()
        mine = [rep[i] for i in order][dp_rank::dp]
        samples = []
        policy.eval()
        for b0 in range(0, len(mine), sbs):
            pids = mine[b0:b0 + sbs]
            txt = torch.cat([embed(p) for p in pids])
            shape = (len(pids),) + lat_shape[1:]
            vids, lats, logps, kls = osp_sample_with_logprob(
                policy, scheduler, vae, shape, txt, dev, wdt, n_steps, g, neg.expand(len(pids), -1, -1),
                sp_group=sp_group, sde_steps=sde_steps, decode=decode)
            lat_st = torch.stack(lats, dim=1)                 # [B, sde+1, C, T, H, W]
            rew, _ = reward_fn(vids if decode else lats[-1].to(dev), [str(p) for p in pids], None)
            samples.append({"pids": pids, "text": txt, "latents": lat_st[:, :-1], "next_latents": lat_st[:, 1:],
                            "log_probs": torch.stack(logps, 1), "rewards": torch.tensor(rew["avg"])})
        # ------------------------------------------------ advantages (gathered over dp ranks)
        local_r = torch.cat([s["rewards"] for s in samples]).float()
        local_p = torch.tensor([p for s in samples for p in s["pids"]])
        if dist.is_initialized() and dp > 1:
            rr = [torch.zeros_like(local_r) for _ in range(W)]
            pp = [torch.zeros_like(local_p) for _ in range(W)]
            dist.all_gather(rr, local_r.to(dev) if dist.get_backend() == "nccl" else local_r)
            dist.all_gather(pp, local_p.to(dev) if dist.get_backend() == "nccl" else local_p)
            all_r = torch.cat([r.cpu() for r in rr[::max(1, gsp)]]).numpy()
            all_p = torch.cat([p.cpu() for p in pp[::max(1, gsp)]]).numpy()
        else:
            all_r, all_p = local_r.numpy(), local_p.numpy()
        if rl.get("per_prompt_stat_tracking", True):
            adv_all = tracker.update([str(p) for p in all_p], all_r)
        else:
            adv_all = (all_r - all_r.mean()) / (all_r.std() + 1e-4)
        n_local = len(local_r)
        adv_local = torch.tensor(adv_all[dp_rank * n_local:(dp_rank + 1) * n_local], dtype=torch.float32)
        if dev.type == "cuda":
            torch.cuda.synchronize()
        t_rollout = _time.perf_counter() - t_epoch
        # ------------------------------------------------ policy update
        policy.train()
        off = 0
        info = {}
        for s in samples:
            B_ = len(s["pids"])
            adv = adv_local[off:off + B_].to(dev)
            off += B_
            for j in range(train_steps):
                smp = {"latents": s["latents"].to(dev), "next_latents": s["next_latents"].to(dev)}
                _, lp, _, _, _ = compute_log_prob_for_training(
                    policy, smp, j, s["text"], wdt, sigmas, n_steps,
                    g if rl.get("use_cfg_in_train", True) else 1.0, neg.expand(B_, -1, -1), sp_group)
                loss, info = grpo_loss(lp, s["log_probs"][:, j].to(dev), adv, rl.get("clip_range", 5e-3),
                                       rl.get("adv_clip_max", 5.0))
                (loss / train_steps).backward()
            opt.grad_scale = clipper.adaptive_clip(lora_params, apply=False)
            opt.step()
            opt.zero_grad(set_to_none=True)
            global_step += 1
            if ema is not None:
                ema.update(policy, global_step)
        if dev.type == "cuda":
            torch.cuda.synchronize()
        t_total = _time.perf_counter() - t_epoch
        log_on_main_process(logger, json.dumps({
            "epoch": epoch, "global_step": global_step, "rollout_s": round(t_rollout, 3),
            "train_s": round(t_total - t_rollout, 3), "epoch_s": round(t_total, 3),
            "reward_mean": float(np.mean(all_r)),
            "reward_std": float(np.std(all_r)), **{k_: float(v) for k_, v in info.items()}}))
        if (epoch + 1) % config.get("save_interval", 100) == 0 or epoch + 1 == epochs:
            path = save_lora(policy, out_dir, global_step)
            if ema is not None:
                save_lora(policy, out_dir, global_step, "-ema", ema)
            if rank == 0:
                clipper.save(path)
                with open(os.path.join(path, RL_STATE), "w") as f:
                    json.dump({"global_step": global_step, "next_epoch": epoch + 1}, f)
    return policy


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    a = ap.parse_args()
    main(load_config(a.config))
    if dist.is_initialized():
        dist.destroy_process_group()
