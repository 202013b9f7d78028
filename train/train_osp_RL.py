"""Mix-GRPO + LoRA reinforcement learning of the OSP-Next DiT (reference: train/train_osp_RL.py:612-1725).

``torchrun --nproc-per-node N train/train_osp_RL.py --config configs/train/osp_14b_RL.yaml``

Per epoch, as in the reference:
  rollout   prompts drawn so each appears ``num_image_per_prompt`` times across the
            data-parallel ranks; ``num_batches_per_epoch`` × ``sample_time_per_prompt``
            rollout batches of ``sample_batch_size``; CFG sampling with SDE steps for
            ``i < sde_steps`` (log-probs and latents stored) and ODE steps after; with
            ``kl_reward > 0`` the KL of each SDE step to the adapter-disabled model
            (reference :229-263) is recorded and subtracted from the logged reward;
  reward    ``multi_score`` (VideoAlign on decoded video, or the latent MLP scorer),
            gathered over data-parallel ranks; ``zero_std_ratio`` of the prompt groups;
  advantage per-prompt mean/std (PerPromptStatTracker, cleared every epoch) or global;
            samples whose advantage is zero are dropped and the kept count is padded to a
            multiple of ``num_batches_per_epoch · sample_time_per_prompt`` (:1389-1404);
  update    ``num_inner_epochs`` passes (:1410), each over a permutation of the kept
            samples (shared inside an SP group) in micro-batches of ``train_batch_size``;
            for every trained SDE step: log-prob under the current policy (CFG via lerp),
            PPO-clip loss plus ``kl_beta`` × KL to the adapter-disabled model (:1468-1498),
            backward; an optimizer step (adaptive clip + fused AdamW over the LoRA
            parameters, LoRA-only EMA) every ``gradient_accumulation_steps`` ×
            ``num_train_timesteps`` backward calls, and one for the remainder;
  save      LoRA (+EMA) ``lora-checkpoint-{step}/adapter_model.bin`` (PEFT key names),
            clipper state and ``rl_training_state.json``; resume from ``lora_config.lora_path``
            with ``resume_epoch`` / ``resume_lr`` / ``resume_override_lr`` (:955-1000);
  eval      every ``eval_freq`` optimizer steps: deterministic (ODE) sampling of the eval
            prompts with the EMA weights swapped in (:1600-1694); latents (and decoded videos
            with a VAE) are written under ``output_dir/eval``.
With ``fsdp_size > 1`` the policy (base + LoRA) is FSDP2-sharded like the reference
(:869-879).  Prompts may be random text embeddings (``rl_config.synthetic_prompts``), the
BASELINE configuration.  Metrics go to ``metrics_file`` (JSONL) and wandb when enabled.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from collections import defaultdict
from typing import Dict, List

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from osp_next_b200 import ops  # noqa: E402
from osp_next_b200.engine import builders as B  # noqa: E402
from osp_next_b200.models.lora import LoraModel  # noqa: E402
from osp_next_b200.parallel.dist_utils import setup_distributed_env  # noqa: E402
from osp_next_b200.parallel.ema import FSDPEMAModel  # noqa: E402
from osp_next_b200.parallel.optim import FusedAdamW  # noqa: E402
from osp_next_b200.parallel.sp import attach_sp  # noqa: E402
from osp_next_b200.rewards import multi_score  # noqa: E402
from osp_next_b200.rl.grpo import (PerPromptStatTracker, calculate_zero_std_ratio,  # noqa: E402
                                   compute_log_prob_for_training, grpo_loss, osp_sample_deterministic,
                                   osp_sample_with_logprob, shifted_sigmas)
from osp_next_b200.utils.clip_grads import AdaptiveGradClipper  # noqa: E402
from osp_next_b200.utils.config import load_config  # noqa: E402
from osp_next_b200.utils.log_utils import MetricsLogger, get_logger, log_on_main_process  # noqa: E402
from osp_next_b200.utils.random_utils import set_seed  # noqa: E402
from osp_next_b200.utils.utils import to_dtype  # noqa: E402

LORA_PREFIX = "lora-checkpoint-"
RL_STATE = "rl_training_state.json"


class AdapterDisabled:
    """The policy with its LoRA branches switched off: the frozen reference model of the
    KL terms, sharing the base weights (no second copy of the network)."""

    def __init__(self, policy: LoraModel):
        self.policy = policy

    def __call__(self, *a, **k):
        with self.policy.disable_adapter():
            return self.policy(*a, **k)


def rl_settings(config) -> dict:
    """rl_config knobs with the reference's names and defaults (train_osp_RL.py:640-690)."""
    rl = config.get("rl_config", {})
    n_steps = rl.get("num_inference_steps", 16)
    sde = rl.get("sde_steps", n_steps)
    s = dict(
        num_inference_steps=n_steps, sde_steps=sde, guidance_scale=rl.get("guidance_scale", 5.0),
        k=rl.get("num_image_per_prompt", 4), sample_batch_size=rl.get("sample_batch_size", 1),
        num_batches_per_epoch=rl.get("num_batches_per_epoch", 1),
        sample_time_per_prompt=rl.get("sample_time_per_prompt", 1),
        train_batch_size=rl.get("train_batch_size", rl.get("sample_batch_size", 1)),
        num_inner_epochs=rl.get("num_inner_epochs", 1),
        num_train_timesteps=max(1, int(sde * rl.get("timestep_fraction", 1.0))),
        clip_range=rl.get("clip_range", 1e-4), adv_clip_max=rl.get("adv_clip_max", 5.0),
        kl_beta=rl.get("kl_beta", 0.0), kl_reward=rl.get("kl_reward", 0.0),
        use_cfg_in_train=rl.get("use_cfg_in_train", True),
        per_prompt_stat_tracking=rl.get("per_prompt_stat_tracking", True), global_std=rl.get("global_std", False),
        eval_freq=rl.get("eval_freq", 10000), eval_num_steps=rl.get("eval_num_steps", 50),
        num_eval_prompts=rl.get("num_eval_prompts", 0),
        height=rl.get("height", 480), width=rl.get("width", 832), num_frames=rl.get("num_frames", 33),
        synthetic=rl.get("synthetic_prompts", rl.get("prompt_file") is None),
        prompt_file=rl.get("prompt_file"), eval_prompt_file=rl.get("eval_prompt_file"),
        num_prompts=rl.get("num_prompts", 64), reward_fn=rl.get("reward_fn", {"latent_mlp": 1.0}),
        gradient_accumulation_steps=config.get("gradient_accumulation_steps", 1),
    )
    s["accum_steps_total"] = s["gradient_accumulation_steps"] * s["num_train_timesteps"]
    return s


def lora_dir(out_dir, step, suffix=""):
    return os.path.join(out_dir, f"{LORA_PREFIX}{step}{suffix}")


def save_lora(policy: LoraModel, out_dir, step, suffix="", ema=None):
    """Every rank takes part (FSDP gathers the shards); rank 0 writes."""
    path = lora_dir(out_dir, step, suffix)
    if ema is not None:
        ema.store(policy)
        ema.ema_copy_to_model(policy)
    policy.save_pretrained(path, write=B.rank() == 0)
    if ema is not None:
        ema.restore(policy)
    return path


def save_rl_state(path, global_step, next_epoch):
    if B.rank() == 0:
        os.makedirs(path, exist_ok=True)
        tmp = os.path.join(path, RL_STATE + ".tmp")
        with open(tmp, "w", encoding="ascii") as f:
            json.dump({"global_step": int(global_step), "next_epoch": int(next_epoch)}, f, indent=2)
        os.replace(tmp, os.path.join(path, RL_STATE))
    if dist.is_initialized():
        dist.barrier()


def load_rl_state(path):
    p = os.path.join(path, RL_STATE)
    if not os.path.exists(p):
        return None
    with open(p, encoding="ascii") as f:
        return json.load(f)


def resume_point(lora_path, resume_epoch, logger):
    """(start_epoch, global_step) from ``rl_training_state.json`` beside the adapter, with
    ``resume_epoch`` overriding the stored epoch (reference :955-1000)."""
    st = load_rl_state(lora_path) if lora_path else None
    step = int(st.get("global_step", 0)) if st else 0
    if resume_epoch is not None:
        if st is None:
            log_on_main_process(logger, f"resume_epoch={resume_epoch} without {RL_STATE}: starting from that epoch")
        return int(resume_epoch), step
    return (int(st.get("next_epoch", 0)) if st else 0), step


def select_samples(adv: torch.Tensor, num_batches_total: int, gen: torch.Generator) -> torch.Tensor:
    """Boolean mask of the samples to train on: non-zero advantage, padded with randomly
    chosen zero-advantage samples up to a multiple of ``num_batches_total``; if nothing is
    left every sample is kept (reference :1387-1404)."""
    mask = adv.abs().sum(dim=1) != 0 if adv.dim() > 1 else adv.abs() != 0
    kept = int(mask.sum())
    if kept == 0:
        return torch.ones_like(mask)
    rem = kept % num_batches_total
    if rem:
        idle = torch.where(~mask)[0]
        need = num_batches_total - rem
        if len(idle) >= need:
            mask[idle[torch.randperm(len(idle), generator=gen)[:need]]] = True
    return mask


def gather_dp(x: torch.Tensor, dp: int, gsp: int, dev) -> torch.Tensor:
    """Concatenate a per-rank tensor over the data-parallel ranks (one rank per SP group)."""
    if not (dist.is_initialized() and dp > 1):
        return x
    t = x if "gloo" in str(dist.get_backend()) else x.to(dev)     # gloo carries CPU tensors
    parts = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t.contiguous())
    return torch.cat([p.cpu() for p in parts[::max(1, gsp)]])


def main(config):
    logger = get_logger()
    setup_distributed_env(timeout_s=config.get("timeout_s", 600))
    rank, W = B.rank(), B.world()
    dev = B.device()
    wdt = to_dtype(config.get("weight_dtype", "bf16"))
    seed = config.get("seed", 42)
    S = rl_settings(config)
    lc = config.get("lora_config", {})
    oc = config.get("optimizer_config", {})
    mcfg = config.get("model_config", {})
    out_dir = config.get("output_dir", "./output_rl_lora")
    os.makedirs(out_dir, exist_ok=True)
    metrics = MetricsLogger(config.get("metrics_file", os.path.join(out_dir, "metrics.jsonl")),
                            use_wandb=config.get("use_wandb", False), run_name=config.get("run_name"))

    sp_rt = B.build_sp(config, mcfg.get("num_heads", 16))
    gsp = sp_rt.spec.world
    dp, dp_rank = max(1, W // gsp), rank // max(1, gsp)
    set_seed(seed + dp_rank)
    sp_group = sp_rt.global_sp_group if gsp > 1 else None

    # ------------------------------------------------------------ model + LoRA (+ FSDP2)
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
        policy.load_adapter(lc["lora_path"])            # before sharding: plain tensors
    for n, p in policy.named_parameters():
        if "lora_" in n:
            p.data = p.data.float()
    shard_group = None
    if W > 1 and config.get("fsdp_size", 1) > 1 and dist.is_initialized():
        mesh = B.build_fsdp_mesh(config)
        B.fsdp_wrap(model, config, mesh, wdt)
        shard_group = (mesh["fsdp"] if "ddp" in (mesh.mesh_dim_names or ()) else mesh).get_group()
    lora_params = [p for n, p in policy.named_parameters() if "lora_" in n]
    ema = FSDPEMAModel(policy, config.get("ema_decay", 0.9999), config.get("ema_update_interval", 1),
                       lora_only=True) if config.get("ema_decay", 0) else None
    opt = FusedAdamW(lora_params, lr=oc.get("lr", 1e-5), betas=tuple(oc.get("betas", (0.9, 0.999))),
                     eps=oc.get("eps", 1e-8), weight_decay=oc.get("weight_decay", 1e-4))
    clipper = AdaptiveGradClipper(init_max_grad_norm=config.get("init_max_grad_norm", 1.0),
                                  model_parallel_group=shard_group)
    ref_model = AdapterDisabled(policy)
    start_epoch, global_step = resume_point(lc.get("lora_path"), config.get("resume_epoch"), logger)
    if lc.get("lora_path"):
        clipper.load(lc["lora_path"])
        lr_over = oc.get("resume_lr") if oc.get("resume_lr") is not None else (
            oc.get("lr", 1e-5) if oc.get("resume_override_lr", False) else None)
        if lr_over is not None:
            for g_ in opt.param_groups:
                g_["lr"] = lr_over

    # ------------------------------------------------------------ rollout setup
    scheduler = B.build_scheduler(config)
    n_steps, g = S["num_inference_steps"], S["guidance_scale"]
    k, sbs = S["k"], S["sample_batch_size"]
    lat_shape = (sbs, mcfg.get("in_dim", 16), (S["num_frames"] - 1) // 4 + 1, S["height"] // 8, S["width"] // 8)
    text_len = mcfg.get("text_len", 512)
    reward_fn = multi_score(dev, S["reward_fn"])
    decode = "videoalign" in S["reward_fn"]
    vae = B.build_vae(config, dev) if (decode or config.get("vae_config", {}).get("vae_path")) else None
    t5 = None if S["synthetic"] else B.build_text_encoder(config, dev)
    prompts = eval_prompts = None
    if not S["synthetic"]:
        with open(S["prompt_file"], encoding="utf-8") as fh:
            prompts = [l.strip() for l in fh if l.strip()]
        if S["eval_prompt_file"]:
            with open(S["eval_prompt_file"], encoding="utf-8") as fh:
                eval_prompts = [l.strip() for l in fh if l.strip()]
    neg = torch.zeros(1, text_len, 4096, dtype=wdt, device=dev)
    sigmas = shifted_sigmas(n_steps, getattr(scheduler, "shift", 1.0), dev)
    tracker = PerPromptStatTracker(S["global_std"]) if S["per_prompt_stat_tracking"] else None
    T = S["num_train_timesteps"]

    def embed(pid, eval_set=False):
        if S["synthetic"]:
            gen = torch.Generator().manual_seed((20_000 if eval_set else 10_000) + pid)
            return torch.randn(1, text_len, 4096, generator=gen).to(dev, wdt)
        return t5([(eval_prompts if eval_set else prompts)[pid]]).to(wdt)

    def check(where):
        ops.check_device_errors_all_ranks(dev, where=where)

    epochs = config.get("num_epochs", 1000)
    save_interval = config.get("save_interval", 100)
    last_done = start_epoch - 1
    for epoch in range(start_epoch, epochs):
        if dev.type == "cuda":
            torch.cuda.synchronize()
        t_epoch = time.perf_counter()
        # ------------------------------------------------ rollout
        gen = torch.Generator().manual_seed(seed + epoch)
        m = max(1, (dp * sbs * S["num_batches_per_epoch"]) // k)
        pool_n = S["num_prompts"] if S["synthetic"] else len(prompts)
        pool = torch.randperm(pool_n, generator=gen)[:m].tolist()
        rep = [p for p in pool for _ in range(k)]
        order = torch.randperm(len(rep), generator=gen).tolist()
        mine = [rep[i] for i in order][dp_rank::dp]
        batches: List[Dict[str, torch.Tensor]] = []
        policy.eval()
        for b0 in range(0, len(mine), sbs):
            pids = mine[b0:b0 + sbs]
            txt = torch.cat([embed(p) for p in pids])
            shape = (len(pids),) + lat_shape[1:]
            for _ in range(S["sample_time_per_prompt"]):
                vids, lats, logps, kls = osp_sample_with_logprob(
                    policy, scheduler, vae, shape, txt, dev, wdt, n_steps, g, neg.expand(len(pids), -1, -1),
                    kl_reward=S["kl_reward"], sp_group=sp_group, sde_steps=S["sde_steps"],
                    ref_model=ref_model if S["kl_reward"] > 0 else None, decode=decode)
                lat_st = torch.stack(lats, dim=1)                 # [B, sde+1, C, T, H, W]
                rew, _ = reward_fn(vids if decode else lats[-1].to(dev), [str(p) for p in pids], None)
                batches.append({"pids": torch.tensor(pids), "text": txt.cpu(), "latents": lat_st[:, :-1],
                                "next_latents": lat_st[:, 1:], "log_probs": torch.stack(logps, 1),
                                "kl": torch.stack(kls, 1), "rewards": torch.as_tensor(rew["avg"]).float()})
        samples = {key: torch.cat([b[key] for b in batches]) for key in batches[0]}
        check(f"RL rollout, epoch {epoch}")
        # ------------------------------------------------ rewards, advantages
        all_r = gather_dp(samples["rewards"], dp, gsp, dev).numpy()
        all_p = gather_dp(samples["pids"], dp, gsp, dev).numpy()
        all_kl = gather_dp(samples["kl"].float(), dp, gsp, dev)
        zero_std = calculate_zero_std_ratio([str(p) for p in all_p], all_r)
        if tracker is not None:
            adv_all = tracker.update([str(p) for p in all_p], all_r)
            tracker.clear()
        else:
            adv_all = (all_r - all_r.mean()) / (all_r.std() + 1e-4)
        adv_all = torch.as_tensor(adv_all).float()
        n_local = len(samples["rewards"])
        adv = adv_all[dp_rank * n_local:(dp_rank + 1) * n_local]
        samples["advantages"] = adv.unsqueeze(1).expand(-1, T).contiguous()
        del samples["rewards"]
        mask = select_samples(samples["advantages"], S["num_batches_per_epoch"] * S["sample_time_per_prompt"],
                              torch.Generator().manual_seed(seed * 7919 + epoch))
        samples = {key: v[mask] for key, v in samples.items()}
        n_kept = len(samples["advantages"])
        shaped_r = all_r[:, None] - S["kl_reward"] * all_kl.numpy().mean(axis=1, keepdims=True)
        metrics.log({"epoch": epoch, "reward_mean": float(all_r.mean()), "reward_std": float(all_r.std()),
                     "reward_max": float(all_r.max()), "reward_min": float(all_r.min()),
                     "reward_kl_shaped_mean": float(shaped_r.mean()), "kl": float(all_kl.mean()),
                     "kl_abs": float(all_kl.abs().mean()), "zero_std_ratio": zero_std,
                     "advantage_mean": float(adv_all.mean()), "advantage_std": float(adv_all.std()),
                     "advantage_abs_mean": float(adv_all.abs().mean()), "samples_kept": n_kept,
                     "samples_total": n_local}, step=global_step)
        if dev.type == "cuda":
            torch.cuda.synchronize()
        t_rollout = time.perf_counter() - t_epoch
        # ------------------------------------------------ policy update
        backward_calls = 0
        info = defaultdict(list)

        def optimizer_step():
            nonlocal global_step, info
            opt.grad_scale = clipper.adaptive_clip(lora_params, apply=False)
            opt.step()
            opt.zero_grad(set_to_none=True)
            global_step += 1
            if ema is not None:
                ema.update(policy, global_step)
            rec = {key: float(torch.stack(v).float().mean()) for key, v in info.items()}
            rec.update(epoch=epoch, grad_norm=float(clipper.grad_norm_before_clip or 0.0),
                       max_grad_norm=float(clipper.max_grad_norm), lr=opt.param_groups[0]["lr"])
            metrics.log(rec, step=global_step)
            info = defaultdict(list)

        for inner in range(S["num_inner_epochs"]):
            policy.train()
            perm = torch.randperm(n_kept, generator=torch.Generator().manual_seed(seed + 1009 * epoch + inner))
            if sp_group is not None:        # the ranks of an SP group hold the same samples
                pt = perm.to(dev) if dev.type == "cuda" else perm
                dist.broadcast(pt, src=dist.get_global_rank(sp_group, 0), group=sp_group)
                perm = pt.cpu()
            shuffled = {key: v[perm] for key, v in samples.items()}
            tbs = max(1, S["train_batch_size"])
            for mb0 in range(0, n_kept, tbs):
                mb = {key: v[mb0:mb0 + tbs] for key, v in shuffled.items()}
                Bm = len(mb["advantages"])
                txt = mb["text"].to(dev)
                neg_b = neg.expand(Bm, -1, -1) if S["use_cfg_in_train"] else None
                g_train = g if S["use_cfg_in_train"] else 1.0
                smp = {"latents": mb["latents"].to(dev), "next_latents": mb["next_latents"].to(dev)}
                for j in range(T):
                    _, lp, mean, std, sqdt = compute_log_prob_for_training(
                        policy, smp, j, txt, wdt, sigmas, n_steps, g_train, neg_b, sp_group)
                    kl = None
                    if S["kl_beta"] > 0:
                        with torch.no_grad():
                            _, _, ref_mean, _, _ = compute_log_prob_for_training(
                                ref_model, smp, j, txt, wdt, sigmas, n_steps, g_train, neg_b, sp_group)
                        var = (std * sqdt) ** 2
                        kl = ((mean - ref_mean) ** 2).mean(dim=tuple(range(1, mean.ndim))) / (2 * var.reshape(-1))
                    loss, step_info = grpo_loss(lp, mb["log_probs"][:, j].to(dev), mb["advantages"][:, j].to(dev),
                                                S["clip_range"], S["adv_clip_max"], kl=kl, kl_beta=S["kl_beta"])
                    (loss / S["accum_steps_total"]).backward()
                    for key, v in step_info.items():
                        info[key].append(v)
                    info["loss"].append(loss.detach())
                    if kl is not None:
                        info["kl_loss"].append(kl.mean().detach())
                    backward_calls += 1
                    if backward_calls % S["accum_steps_total"] == 0:
                        optimizer_step()
        if backward_calls % S["accum_steps_total"] != 0:
            optimizer_step()
        check(f"RL update, epoch {epoch}")
        if dev.type == "cuda":
            torch.cuda.synchronize()
        t_total = time.perf_counter() - t_epoch
        metrics.log({"epoch": epoch, "rollout_s": round(t_rollout, 3), "train_s": round(t_total - t_rollout, 3),
                     "epoch_s": round(t_total, 3)}, step=global_step)
        log_on_main_process(logger, json.dumps({
            "epoch": epoch, "global_step": global_step, "rollout_s": round(t_rollout, 3),
            "train_s": round(t_total - t_rollout, 3), "reward_mean": float(all_r.mean()),
            "zero_std_ratio": zero_std, "samples_kept": n_kept}))
        # ------------------------------------------------ save
        if epoch > 0 and epoch % save_interval == 0:
            path = save_lora(policy, out_dir, global_step)
            if ema is not None:
                save_lora(policy, out_dir, global_step, "-ema", ema)
            if rank == 0:
                clipper.save(path)
            save_rl_state(path, global_step, epoch + 1)
        last_done = epoch
        # ------------------------------------------------ eval (EMA weights, deterministic sampling)
        n_eval = S["num_eval_prompts"] or (len(eval_prompts) if eval_prompts else 0)
        if n_eval and global_step > 0 and global_step % S["eval_freq"] == 0:
            evaluate(policy, ema, scheduler, vae, embed, n_eval, lat_shape, dev, wdt, S, neg, out_dir, global_step,
                     dp, dp_rank, metrics)
    # ---------------------------------------------------- final save
    completed = max(start_epoch, last_done + 1)
    path = save_lora(policy, out_dir, global_step)
    if ema is not None:
        save_lora(policy, out_dir, global_step, "-ema", ema)
    if rank == 0:
        clipper.save(path)
    save_rl_state(path, global_step, completed)
    metrics.close()
    return policy


@torch.no_grad()
def evaluate(policy, ema, scheduler, vae, embed, n_eval, lat_shape, dev, wdt, S, neg, out_dir, step, dp, dp_rank,
             metrics):
    """Deterministic sampling of the eval prompts with the EMA LoRA weights (reference
    :1600-1694); each data-parallel rank takes every dp-th prompt and writes its latents
    (and, with a VAE, mp4 videos) under ``out_dir/eval/step_{step}``."""
    policy.eval()
    if ema is not None:
        ema.store(policy)
        ema.ema_copy_to_model(policy)
    edir = os.path.join(out_dir, "eval", f"step_{step}")
    os.makedirs(edir, exist_ok=True)
    t0 = time.perf_counter()
    for pid in range(dp_rank, n_eval, dp):
        txt = embed(pid, eval_set=True)
        shape = (1,) + lat_shape[1:]
        gen = torch.Generator(device=dev).manual_seed(pid) if dev.type == "cuda" else torch.Generator().manual_seed(pid)
        out = osp_sample_deterministic(policy, scheduler, vae, shape, txt, dev, wdt, S["eval_num_steps"],
                                       S["guidance_scale"], neg, decode=vae is not None, generator=gen)
        if vae is not None:
            from osp_next_b200.data.utils.video_io import save_video
            vid = ((out[0].float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(1, 2, 3, 0).cpu()
            save_video(vid, os.path.join(edir, f"eval_{pid:04d}.mp4"), fps=16)
        else:
            torch.save(out.cpu(), os.path.join(edir, f"eval_{pid:04d}_latent.pt"))
    if ema is not None:
        ema.restore(policy)
    ops.check_device_errors_all_ranks(dev, where=f"RL eval at step {step}")
    metrics.log({"eval_s": round(time.perf_counter() - t0, 3), "eval_prompts": n_eval}, step=step)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    a = ap.parse_args()
    main(load_config(a.config))
    if dist.is_initialized():
        dist.destroy_process_group()
