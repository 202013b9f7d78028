"""Mix-GRPO: SDE sampling with log-probabilities, per-prompt advantages, clipped loss.

Reference: train/train_osp_RL.py — ``sde_step_with_logprob`` (67-129),
``osp_sample_with_logprob`` (132-285), ``osp_sample_deterministic`` (288-364),
``compute_log_prob_for_training`` (367-417), ``DistributedKRepeatSampler``
(449-487), ``PerPromptStatTracker`` (490-516), ``calculate_zero_std_ratio``
(519-530), policy loss (1485-1503).  Same formulas; on CUDA the SDE step is one
fused kernel (:func:`osp_next_b200.ops.sde_step`), and cond/uncond run as one
batch of 2 through the fused DiT path.  The SDE window is the fixed prefix
``i < sde_steps`` as in the reference.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist

from .. import ops


def shifted_sigmas(num_steps: int, shift: float, device="cpu") -> torch.Tensor:
    """σ schedule of the RL trainer: linspace(1, 0) then ``shift·σ/(1+(shift−1)σ)``
    when shift ≠ 1 (train_osp_RL.py:160-163)."""
    s = torch.linspace(1.0, 0.0, num_steps + 1, device=device)
    if shift != 1.0:
        s = shift * s / (1 + (shift - 1) * s)
    return s


def sde_step_with_logprob(sigmas, model_output, timestep_index, sample, num_inference_steps, prev_sample=None,
                          generator=None, determistic=False, return_dt_and_std_dev_t=False, sp_group=None,
                          noise=None, use_kernel=True):
    """One Mix-GRPO step; returns (prev_sample, log_prob[B], prev_mean, std·sqrt(−dt)) like the reference.

    ``noise`` lets callers pass the Gaussian draw explicitly (tests, SP broadcast).
    """
    model_output = model_output.float()
    sample = sample.float()
    sigma = sigmas[timestep_index]
    sigma_prev = sigmas[timestep_index + 1]
    smax = float(sigmas[0])
    smin = float(sigmas[-1])
    dt = sigma_prev - sigma
    if prev_sample is not None and generator is not None:
        raise ValueError("Cannot pass both generator and prev_sample.")
    if prev_sample is None and not determistic and timestep_index < num_inference_steps - 1 and noise is None:
        noise = torch.randn(model_output.shape, generator=generator, device=model_output.device,
                            dtype=model_output.dtype)
        if sp_group is not None:
            dist.broadcast(noise, src=dist.get_global_rank(sp_group, 0), group=sp_group)
    if (use_kernel and sample.is_cuda and not determistic and not return_dt_and_std_dev_t
            and not torch.is_grad_enabled() and sample[0].numel() >= 512):
        prev, logp, mean = ops.sde_step(sample, model_output, float(sigma), float(dt), smin, smax,
                                        noise=noise if prev_sample is None else None,
                                        prev_sample=prev_sample)
        std = (smin + (smax - smin) * float(sigma)) * math.sqrt(-float(dt))
        return prev, logp, mean, torch.full((), std, device=sample.device)
    sigma_b = sigma.view(-1, *([1] * (sample.ndim - 1))) if torch.is_tensor(sigma) else torch.tensor(sigma)
    dt_b = dt.view(-1, *([1] * (sample.ndim - 1))) if torch.is_tensor(dt) else torch.tensor(dt)
    std_dev_t = smin + (smax - smin) * sigma_b
    prev_mean = (sample * (1 + std_dev_t ** 2 / (2 * sigma_b) * dt_b)
                 + model_output * (1 + std_dev_t ** 2 * (1 - sigma_b) / (2 * sigma_b)) * dt_b)
    if prev_sample is None:
        if timestep_index < num_inference_steps - 1 and noise is not None:
            prev_sample = prev_mean + std_dev_t * torch.sqrt(-1 * dt_b) * noise
        else:
            prev_sample = prev_mean
    else:
        prev_sample = prev_sample.float()
    if determistic:
        prev_sample = sample + dt_b * model_output
    sd = std_dev_t * torch.sqrt(-1 * dt_b)
    log_prob = (-((prev_sample.detach() - prev_mean) ** 2) / (2 * sd ** 2) - torch.log(sd)
                - torch.log(torch.sqrt(2 * torch.as_tensor(math.pi))))
    log_prob = log_prob.mean(dim=tuple(range(1, log_prob.ndim)))
    if return_dt_and_std_dev_t:
        return prev_sample, log_prob, prev_mean, std_dev_t, torch.sqrt(-1 * dt_b)
    return prev_sample, log_prob, prev_mean, sd


def _cfg_predict(model, latents, t, text, neg, guidance):
    """Velocity with CFG: cond/uncond as one batch of 2 (fused path) or a single pass."""
    B = latents.shape[0]
    tb = t.expand(B).to(latents.device)
    if guidance > 1.0 and neg is not None:
        pred = model(torch.cat([latents, latents]), torch.cat([tb, tb]), torch.cat([text, neg]))
        c, u = pred[:B].float(), pred[B:].float()
        return u + guidance * (c - u)
    return model(latents, tb, text).float()


@torch.no_grad()
def osp_sample_with_logprob(model, scheduler, vae, latent_shape, text_embeddings, device, weight_dtype,
                            num_inference_steps=50, guidance_scale=5.0, negative_text_embeddings=None,
                            determistic=False, kl_reward=0.0, sp_group=None, sde_steps=None, ref_model=None,
                            decode=True, generator=None):
    """Rollout: SDE steps for ``i < sde_steps`` (log-probs recorded), ODE afterwards."""
    if sde_steps is None:
        sde_steps = num_inference_steps
    B = latent_shape[0]
    latents = torch.randn(latent_shape, device=device, dtype=torch.float32, generator=generator)
    if sp_group is not None:
        dist.broadcast(latents, src=dist.get_global_rank(sp_group, 0), group=sp_group)
    shift = getattr(scheduler, "shift", 1.0)
    sigmas = shifted_sigmas(num_inference_steps, shift, device)
    timesteps = sigmas * 1000.0
    all_latents, all_log_probs, all_kl = [latents], [], []
    for i in range(num_inference_steps):
        is_sde = i < sde_steps
        x_in = latents.to(weight_dtype)
        v = _cfg_predict(model, x_in, timesteps[i], text_embeddings, negative_text_embeddings, guidance_scale)
        lat_prev = latents
        latents, log_prob, mean, std = sde_step_with_logprob(sigmas, v, i, latents, num_inference_steps,
                                                             determistic=not is_sde, sp_group=sp_group,
                                                             generator=generator)
        if is_sde:
            all_latents.append(latents)
            all_log_probs.append(log_prob)
            if kl_reward > 0 and not determistic and ref_model is not None:
                v_ref = _cfg_predict(ref_model, lat_prev.to(weight_dtype), timesteps[i], text_embeddings,
                                     negative_text_embeddings, guidance_scale)
                _, _, ref_mean, _ = sde_step_with_logprob(sigmas, v_ref, i, lat_prev, num_inference_steps,
                                                          prev_sample=latents, sp_group=sp_group)
                kl = ((mean - ref_mean) ** 2 / (2 * std ** 2)).mean(dim=tuple(range(1, mean.ndim)))
                all_kl.append(kl)
            else:
                all_kl.append(torch.zeros(B, device=device))
    videos = vae.decode(latents) if (decode and vae is not None) else latents
    return videos, [l.cpu() for l in all_latents], [l.cpu() for l in all_log_probs], [k.cpu() for k in all_kl]


@torch.no_grad()
def osp_sample_deterministic(model, scheduler, vae, latent_shape, text_embeddings, device, weight_dtype,
                             num_inference_steps=50, guidance_scale=5.0, negative_text_embeddings=None,
                             decode=True, generator=None):
    latents = torch.randn(latent_shape, device=device, dtype=torch.float32, generator=generator)
    sigmas = shifted_sigmas(num_inference_steps, getattr(scheduler, "shift", 1.0), device)
    timesteps = sigmas * 1000.0
    for i in range(num_inference_steps):
        v = _cfg_predict(model, latents.to(weight_dtype), timesteps[i], text_embeddings, negative_text_embeddings,
                         guidance_scale)
        latents = latents + (sigmas[i + 1] - sigmas[i]) * v
    return vae.decode(latents) if (decode and vae is not None) else latents


def compute_log_prob_for_training(model, sample, step_idx, text_embeddings, weight_dtype, sigmas, num_inference_steps,
                                  guidance_scale=1.0, negative_text_embeddings=None, sp_group=None):
    """Log-prob of the stored next latent under the current policy (grad through cond)."""
    x_in = sample["latents"][:, step_idx].to(weight_dtype)
    t = (sigmas[step_idx] * 1000.0).expand(x_in.shape[0]).to(x_in.device)
    pred = model(x_in, t, text_embeddings)
    if guidance_scale > 1.0 and negative_text_embeddings is not None:
        with torch.no_grad():
            unc = model(x_in, t, negative_text_embeddings).detach()
        pred = torch.lerp(unc.float(), pred.float(), guidance_scale)
    return sde_step_with_logprob(sigmas, pred.float(), step_idx, sample["latents"][:, step_idx].float(),
                                 num_inference_steps, prev_sample=sample["next_latents"][:, step_idx].float(),
                                 return_dt_and_std_dev_t=True, sp_group=sp_group)


def grpo_loss(log_prob, old_log_prob, advantages, clip_range: float, adv_clip_max: float,
              kl: Optional[torch.Tensor] = None, kl_beta: float = 0.0):
    """PPO-clip objective on per-sample log-probs (train_osp_RL.py:1485-1503)."""
    adv = torch.clamp(advantages, -adv_clip_max, adv_clip_max)
    ratio = torch.exp(log_prob - old_log_prob)
    unclipped = -adv * ratio
    clipped = -adv * torch.clamp(ratio, 1.0 - clip_range, 1.0 + clip_range)
    policy_loss = torch.mean(torch.maximum(unclipped, clipped))
    loss = policy_loss + (kl_beta * kl.mean() if (kl is not None and kl_beta > 0) else 0.0)
    info = {
        "approx_kl": 0.5 * torch.mean((log_prob - old_log_prob) ** 2).detach(),
        "clipfrac": torch.mean((torch.abs(ratio - 1.0) > clip_range).float()).detach(),
        "policy_loss": policy_loss.detach(),
    }
    return loss, info


class DistributedKRepeatSampler(torch.utils.data.Sampler):
    """Each of ``m = world·batch/k`` prompts appears ``k`` times across the world per step."""

    def __init__(self, dataset, batch_size, k, num_replicas, rank, seed=0):
        self.dataset = dataset
        self.batch_size = batch_size
        self.k = k
        self.num_replicas = num_replicas
        self.rank = rank
        self.seed = seed
        self.total_samples = num_replicas * batch_size
        if self.total_samples % k != 0:
            raise ValueError(f"k cannot divide n*b, k={k}, num_replicas={num_replicas}, batch_size={batch_size}")
        self.m = self.total_samples // k
        self.epoch = 0

    def __iter__(self):
        while True:
            g = torch.Generator()
            g.manual_seed(self.seed + self.epoch)
            idx = torch.randperm(len(self.dataset), generator=g)[: self.m].tolist()
            rep = [i for i in idx for _ in range(self.k)]
            perm = torch.randperm(len(rep), generator=g).tolist()
            shuffled = [rep[i] for i in perm]
            s = self.rank * self.batch_size
            yield shuffled[s: s + self.batch_size]

    def set_epoch(self, epoch):
        self.epoch = epoch


class PerPromptStatTracker:
    """Advantages normalised by each prompt's running reward statistics."""

    def __init__(self, global_std=False):
        self.global_std = global_std
        self.stats: Dict[str, list] = {}
        self.history_prompts = set()

    def update(self, prompts, rewards):
        prompts = np.array(prompts)
        rewards = np.array(rewards, dtype=np.float64)
        unique = np.unique(prompts)
        adv = np.zeros_like(rewards)
        for p in unique:
            self.stats.setdefault(p, [])
            self.stats[p] = list(self.stats[p]) + list(rewards[prompts == p])
            self.history_prompts.add(hash(p))
        for p in unique:
            hist = np.stack(self.stats[p])
            pr = rewards[prompts == p]
            mean = np.mean(hist, axis=0, keepdims=True)
            std = (np.std(rewards, axis=0, keepdims=True) if self.global_std else np.std(hist, axis=0, keepdims=True))
            adv[prompts == p] = (pr - mean) / (std + 1e-4)
        return adv

    def get_stats(self):
        avg = sum(len(v) for v in self.stats.values()) / len(self.stats) if self.stats else 0
        return avg, len(self.history_prompts)

    def clear(self):
        self.stats = {}


def calculate_zero_std_ratio(prompts: Sequence[str], rewards: np.ndarray) -> float:
    arr = np.array(prompts)
    uniq, inv, counts = np.unique(arr, return_inverse=True, return_counts=True)
    grouped = np.asarray(rewards)[np.argsort(inv, kind="stable")]
    groups = np.split(grouped, np.cumsum(counts)[:-1])
    stds = np.array([np.std(g) for g in groups])
    return float(np.count_nonzero(stds == 0) / len(stds))
