"""Rectified-flow (flow-matching) scheduler.

Same schedules and update rules as the reference (ospnext/schedulers/
flow_matching.py:10-187): σ from a static shift, a resolution-dependent
exponential shift, or logit-normal sampling; ``x_t = σ·n + (1−σ)·x0``; velocity
target ``n − x0``; Euler steps ``x ← x + v·(σ_{i+1} − σ_i)`` with two-pass CFG.
On CUDA the CFG combine and the Euler update are one fused kernel
(:func:`osp_next_b200.ops.cfg_euler_step`), and cond/uncond run as one batch of 2
when the predictor accepts it (``batch_cfg=True``).
"""
from __future__ import annotations

import logging
import math
from typing import Callable, Optional

import torch

from .. import ops


class FlowMatchingScheduler:
    def __init__(self, num_inference_steps=None, guidance_scale=0.0, use_dynamic_shifting=False,
                 use_logitnorm_time_sampling=False, shift=1.0, **kwargs):
        self.num_inference_steps = num_inference_steps
        self.guidance_scale = guidance_scale
        self.do_classifier_free_guidance = guidance_scale > 1.0
        self.use_dynamic_shifting = use_dynamic_shifting
        self.shift = shift
        self.use_logitnorm_time_sampling = use_logitnorm_time_sampling
        if use_dynamic_shifting:
            self.base_image_seq = kwargs.pop("base_image_seq", 256)
            self.max_image_seq = kwargs.pop("max_image_seq", 4096)
            self.base_shift = kwargs.pop("base_shift", 0.5)
            self.max_shift = kwargs.pop("max_shift", 1.15)
            self.shift_k = (self.max_shift - self.base_shift) / (self.max_image_seq - self.base_image_seq)
            self.shift_b = self.base_shift - self.shift_k * self.base_image_seq
        if use_logitnorm_time_sampling:
            self.logit_mean = kwargs.pop("logit_mean", 0.0)
            self.logit_std = kwargs.pop("logit_std", 1.0)
        self._sigma_min = 0.0
        self._sigma_max = 1.0
        self.batch_cfg = kwargs.pop("batch_cfg", True)

    @property
    def sigma_min(self):
        return self._sigma_min

    @property
    def sigma_max(self):
        return self._sigma_max

    # ------------------------------------------------------------------ training
    def interpolation(self, latents, prior_dist, sigmas):
        dt = latents.dtype
        return (sigmas.float() * prior_dist.float() + (1.0 - sigmas.float()) * latents.float()).to(dt)

    def training_losses(self, model_output, latents, prior_dist, mask=None, sigmas=None, **kwargs):
        if mask is not None:
            raise ValueError("mask is not supported currently.")
        target = prior_dist - latents
        loss = torch.nn.functional.mse_loss(model_output.float(), target.float(), reduction="mean")
        loss = loss * self._training_weight(sigmas)
        return [loss]

    def q_sample(self, latents, sigmas=None, prior_dist=None, **kwargs):
        b, c, t, h, w = latents.shape
        if prior_dist is None:
            prior_dist = torch.randn_like(latents)
        image_seq_len = h * w // 4 if self.use_dynamic_shifting else None
        sigmas = self._set_sigmas(sigmas=sigmas, batch_size=b, image_seq_len=image_seq_len, device=latents.device)
        timesteps = sigmas.clone() * 1000
        while sigmas.ndim < latents.ndim:
            sigmas = sigmas.unsqueeze(-1)
        x_t = self.interpolation(latents, prior_dist, sigmas)
        return dict(x_t=x_t, prior_dist=prior_dist, sigmas=sigmas, timesteps=timesteps)

    def _set_sigmas(self, sigmas=None, batch_size=None, image_seq_len=None, training=True,
                    device=torch.device("cpu")):
        if training:
            if sigmas is None:
                if self.use_logitnorm_time_sampling:
                    sigmas = torch.sigmoid(torch.normal(mean=self.logit_mean, std=self.logit_std,
                                                        size=(batch_size,), device=device))
                else:
                    sigmas = torch.rand((batch_size,), device=device)
        else:
            sigmas = torch.linspace(self.sigma_max, self.sigma_min, self.num_inference_steps + 1, device=device)
        if self.use_dynamic_shifting:
            if image_seq_len is None:
                raise ValueError("you have to pass `image_seq_len` when `use_dynamic_shifting` is set to be `True`")
            shift = math.exp(image_seq_len * self.shift_k + self.shift_b)
        else:
            shift = self.shift
        return shift * sigmas / (1 + (shift - 1) * sigmas)

    def _training_weight(self, sigmas):
        return 1.0

    # ------------------------------------------------------------------ sampling
    def sigmas_for_sampling(self, device="cpu"):
        return self._set_sigmas(training=False, device=device)

    def _step(self, model_output, latents, delta_t):
        dt = latents.dtype
        return (latents.float() + model_output.float() * float(delta_t)).to(dt)

    def get_latent_model_input(self, latents, **kwargs):
        return latents, latents

    def sample(self, model, latents, prompt_embeds=None, negative_prompt_embeds=None,
               step_callback: Optional[Callable] = None, cfg_parallel=None, max_steps=None,
               cuda_graph: bool = False, **model_kwargs):
        """Euler sampling with CFG.

        ``cfg_parallel``: optional :class:`osp_next_b200.parallel.cfg.CFGParallel`
        that runs cond on one half of the ranks and uncond on the other.
        ``max_steps``: stop after the first steps of the schedule (timing runs).
        ``cuda_graph``: capture the model call once (after one eager warm-up step) and
        replay it for the remaining steps; single-GPU CUDA inference only.
        """
        n = self.num_inference_steps
        sigmas = self._set_sigmas(training=False)
        timesteps = sigmas.clone() * 1000
        cfg = self.do_classifier_free_guidance and negative_prompt_embeds is not None
        g = self.guidance_scale
        if hasattr(model, "reset_text_kv_cache"):
            model.reset_text_kv_cache()
        graphed = bool(cuda_graph and latents.is_cuda and getattr(model, "parallel", None) is None
                       and cfg_parallel is None)
        if graphed:
            from ..utils.graphs import CUDAGraphRunner
            model = CUDAGraphRunner(model)
        e2 = None
        if cfg and cfg_parallel is None and self.batch_cfg:
            e2 = torch.cat([prompt_embeds, negative_prompt_embeds], 0)
        for i in range(n if max_steps is None else min(n, max_steps)):
            t = timesteps[i]
            dt_sigma = float(sigmas[i + 1] - sigmas[i])
            B = latents.shape[0]
            if cfg and cfg_parallel is not None:
                emb = prompt_embeds if cfg_parallel.is_cond_rank else negative_prompt_embeds
                pred = model(latents, t.expand(B).to(latents.device), emb)
                cond, uncond = cfg_parallel.exchange(pred)
                latents = ops.cfg_euler_step(latents, cond, uncond, g, dt_sigma)
            elif cfg and self.batch_cfg:
                x2 = torch.cat([latents, latents], 0)
                pred = model(x2, t.expand(2 * B).to(latents.device), e2)
                latents = ops.cfg_euler_step(latents, pred[:B], pred[B:], g, dt_sigma)
            elif cfg:
                cond = model(latents, t.expand(B).to(latents.device), prompt_embeds)
                if graphed:                  # the next replay overwrites the static output
                    cond = cond.clone()
                uncond = model(latents, t.expand(B).to(latents.device), negative_prompt_embeds)
                latents = ops.cfg_euler_step(latents, cond, uncond, g, dt_sigma)
            else:
                pred = model(latents, t.expand(B).to(latents.device), prompt_embeds)
                latents = self._step(pred, latents, dt_sigma)
            if step_callback is not None:
                step_callback(i, latents)
        return latents


flow_scheduler = {"flow_matching": FlowMatchingScheduler}
