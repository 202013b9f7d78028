"""Text-to-video sampling pipeline (reference: ospnext/pipelines/t2v_pipeline.py:12-219).

Same call surface: prompt cleaning + tokenisation + T5 encoding (cond and
negative), latent initialisation broadcast inside the SP group, flow-matching
sampling, VAE decode to uint8 ``[b, t, h, w, c]``.  Additions: precomputed
``prompt_embeds`` may live in (pinned) host memory and are copied in
asynchronously; ``output_type="latent"`` skips the VAE; ``cfg_parallel`` splits
cond/uncond across ranks; ``max_steps`` stops after the first steps of the
schedule (used for timing).
"""
from __future__ import annotations

import html
import re
from typing import Optional

import torch
import torch.distributed as dist

from ..parallel.sp_state import sp_state
from ..utils.constant import NEGATIVE_PROMPT


def _fix_text(text: str) -> str:
    try:
        import ftfy
        return ftfy.fix_text(text)
    except Exception:
        return text


class T2VInferencePipeline:
    vae_scale_factor_temporal = 4
    vae_scale_factor_spatial = 8

    def __init__(self, vae=None, tokenizer=None, text_encoder=None, predictor=None, scheduler=None):
        self.vae = vae
        self.tokenizer = tokenizer
        self.text_encoder = text_encoder
        self.predictor = predictor
        self.scheduler = scheduler

    # ------------------------------------------------------------------ text
    @staticmethod
    def prompt_preprocess(prompt: str) -> str:
        text = html.unescape(html.unescape(_fix_text(prompt))).strip()
        return re.sub(r"\s+", " ", text).strip()

    def _get_prompt_embeds(self, prompt, max_sequence_length=512, device=None, dtype=None):
        prompt = [self.prompt_preprocess(p) for p in prompt]
        ids, mask = self.tokenizer(prompt, return_mask=True, add_special_tokens=True)
        emb = self.text_encoder(ids.to(device), mask.to(device))
        return emb.to(dtype)

    def encode_texts(self, prompt, negative_prompt=None, do_classifier_free_guidance=True, prompt_embeds=None,
                     negative_prompt_embeds=None, max_sequence_length=512, device=None, dtype=None):
        prompt = [prompt] if isinstance(prompt, str) else prompt
        batch_size = len(prompt) if prompt is not None else prompt_embeds.shape[0]
        if prompt_embeds is None:
            prompt_embeds = self._get_prompt_embeds(prompt, max_sequence_length, device, dtype)
        if do_classifier_free_guidance and negative_prompt_embeds is None:
            negative_prompt = negative_prompt or ""
            negative_prompt = batch_size * [negative_prompt] if isinstance(negative_prompt, str) else negative_prompt
            if batch_size != len(negative_prompt):
                raise ValueError("negative_prompt batch size must match prompt batch size")
            negative_prompt_embeds = self._get_prompt_embeds(negative_prompt, max_sequence_length, device, dtype)
        return prompt_embeds, negative_prompt_embeds

    # ------------------------------------------------------------------ latents
    def prepare_latents(self, shape, generator, device, dtype, latents=None):
        if latents is None:
            latents = torch.randn(shape, generator=generator, dtype=dtype).to(device)
        else:
            latents = latents.to(device, non_blocking=True)
        if sp_state.is_initialized and sp_state.global_sp_group is not None and sp_state.global_sp_size > 1:
            dist.broadcast(latents, src=dist.get_global_rank(sp_state.global_sp_group, 0),
                           group=sp_state.global_sp_group)
        return latents

    def decode_latents(self, latents, value_range=(-1, 1), normalize=True):
        video = self.vae.decode(latents)
        if normalize:
            low, high = value_range
            video = video.clamp(low, high).sub(low).div(max(high - low, 1e-5))
        return video.mul(255).add_(0.5).clamp_(0, 255).permute(0, 2, 3, 4, 1).to("cpu", torch.uint8)

    @torch.inference_mode()
    def __call__(self, prompt=None, negative_prompt=None, prompt_embeds=None, negative_prompt_embeds=None,
                 num_frames=49, height=480, width=832, seed=None, max_sequence_length=512, device="cuda:0",
                 latents=None, output_type: str = "video", cfg_parallel=None, max_steps: Optional[int] = None,
                 cuda_graph: bool = False):
        if negative_prompt is None or negative_prompt == "":
            negative_prompt = NEGATIVE_PROMPT
        batch_size = 1 if isinstance(prompt, str) else (len(prompt) if prompt is not None else prompt_embeds.shape[0])
        do_cfg = self.scheduler.do_classifier_free_guidance
        emb_dtype = getattr(self.text_encoder, "dtype", torch.bfloat16) if self.text_encoder is not None \
            else (prompt_embeds.dtype if prompt_embeds is not None else torch.bfloat16)
        if prompt_embeds is not None:
            prompt_embeds = prompt_embeds.to(device, non_blocking=True)
        if negative_prompt_embeds is not None:
            negative_prompt_embeds = negative_prompt_embeds.to(device, non_blocking=True)
        prompt_embeds, negative_prompt_embeds = self.encode_texts(
            prompt, negative_prompt, do_cfg, prompt_embeds, negative_prompt_embeds, max_sequence_length, device,
            emb_dtype)
        shape = (batch_size, self.predictor.in_dim, (num_frames - 1) // self.vae_scale_factor_temporal + 1,
                 height // self.vae_scale_factor_spatial, width // self.vae_scale_factor_spatial)
        generator = torch.Generator().manual_seed(seed) if seed is not None else None
        latents = self.prepare_latents(shape, generator, device, prompt_embeds.dtype, latents)
        latents = self.scheduler.sample(self.predictor, latents, prompt_embeds=prompt_embeds,
                                        negative_prompt_embeds=negative_prompt_embeds, cfg_parallel=cfg_parallel,
                                        max_steps=max_steps, cuda_graph=cuda_graph)
        if output_type == "latent" or self.vae is None:
            return latents
        return self.decode_latents(latents.to(self.vae.dtype))


pipeline = {"t2v": T2VInferencePipeline}
