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

import math
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import torch

from .. import ops


@dataclass(frozen=True)
class ShiftRule:
    """Time shift of the flow-matching schedule: σ ↦ s·σ / (1 + (s − 1)·σ).

    ``s`` is either a constant or resolution dependent, ``s = exp(slope·L + intercept)``
    with ``L`` the latent tokens per frame, the line passing through
    (``base_image_seq``, ``base_shift``) and (``max_image_seq``, ``max_shift``) in log space.
    """
    constant: float = 1.0
    log_line: Optional[Tuple[float, float]] = None      # (slope, intercept) of log s against L

    @classmethod
    def through(cls, seq_lo: float, log_s_lo: float, seq_hi: float, log_s_hi: float) -> "ShiftRule":
        slope = (log_s_hi - log_s_lo) / (seq_hi - seq_lo)
        return cls(log_line=(slope, log_s_lo - slope * seq_lo))

    def factor(self, seq_len: Optional[int]) -> float:
        if self.log_line is None:
            return self.constant
        if seq_len is None:
            raise ValueError("a resolution-dependent shift needs image_seq_len (latent tokens per frame)")
        slope, intercept = self.log_line
        return math.exp(slope * seq_len + intercept)

    def __call__(self, sigmas: torch.Tensor, seq_len: Optional[int] = None) -> torch.Tensor:
        s = self.factor(seq_len)
        return s * sigmas / (1 + (s - 1) * sigmas)


class FlowMatchingScheduler:
    """Keyword names follow the reference's YAML configs (``shift``, ``use_dynamic_shifting``
    with ``base_image_seq`` / ``max_image_seq`` / ``base_shift`` / ``max_shift``,
    ``use_logitnorm_time_sampling`` with ``logit_mean`` / ``logit_std``)."""

    def __init__(self, num_inference_steps=None, guidance_scale=0.0, use_dynamic_shifting=False,
                 use_logitnorm_time_sampling=False, shift=1.0, batch_cfg=True, base_image_seq=256,
                 max_image_seq=4096, base_shift=0.5, max_shift=1.15, logit_mean=0.0, logit_std=1.0, **unused):
        self.num_inference_steps = num_inference_steps
        self.guidance_scale = guidance_scale
        self.do_classifier_free_guidance = guidance_scale > 1.0
        self.shift = shift
        self.use_dynamic_shifting = use_dynamic_shifting
        self.use_logitnorm_time_sampling = use_logitnorm_time_sampling
        self.shift_rule = (ShiftRule.through(base_image_seq, base_shift, max_image_seq, max_shift)
                           if use_dynamic_shifting else ShiftRule(constant=shift))
        self.logit_normal = (logit_mean, logit_std) if use_logitnorm_time_sampling else None
        self.batch_cfg = batch_cfg
        self._sigma_min, self._sigma_max = 0.0, 1.0

    @property
    def sigma_min(self):
        return self._sigma_min

    @property
    def sigma_max(self):
        return self._sigma_max

    def draw_training_sigmas(self, batch_size, device=torch.device("cpu")):
        """Unshifted σ per sample: U[0, 1), or sigmoid of N(mean, std) (logit-normal)."""
        if self.logit_normal is None:
            return torch.rand((batch_size,), device=device)
        mean, std = self.logit_normal
        return torch.sigmoid(torch.randn((batch_size,), device=device) * std + mean)

    def inference_grid(self, device=torch.device("cpu")):
        """Unshifted σ of the sampler: num_inference_steps + 1 points from σ_max down to σ_min."""
        return torch.linspace(self._sigma_max, self._sigma_min, self.num_inference_steps + 1, device=device)

    def _set_sigmas(self, sigmas=None, batch_size=None, image_seq_len=None, training=True,
                    device=torch.device("cpu")):
        """Shifted σ: the sampler grid (``training=False``), else the given or freshly drawn σ."""
        if not training:
            base = self.inference_grid(device)
        else:
            base = self.draw_training_sigmas(batch_size, device) if sigmas is None else sigmas
        return self.shift_rule(base, image_seq_len)

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
               cuda_graph: bool = False, check_errors_every: int = 1, **model_kwargs):
        """Euler sampling with CFG.

        ``cfg_parallel``: optional :class:`osp_next_b200.parallel.cfg.CFGParallel`
        that runs cond on one half of the ranks and uncond on the other.
        ``max_steps``: stop after the first steps of the schedule (timing runs).
        ``cuda_graph``: capture the model call once (after one eager warm-up step) and
        replay it for the remaining steps; single-GPU CUDA inference only.
        ``check_errors_every``: every that many steps (and after the last) read the device
        error word and raise :class:`osp_next_b200.ops.DeviceWaitError` if a bounded wait in
        a kernel gave up (e.g. a peer stalled in the NVLink exchange); 0 disables.
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
        n_run = n if max_steps is None else min(n, max_steps)
        for i in range(n_run):
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
            if check_errors_every and latents.is_cuda and ((i + 1) % check_errors_every == 0 or i + 1 == n_run):
                ops.check_device_errors(latents.device, where=f"sampling step {i}")
        return latents


flow_scheduler = {"flow_matching": FlowMatchingScheduler}
