"""VideoAlign reward model (reference: ospnext/rewards/videoalign_model.py:124-429,
videoalign_inference.py:43-249, videoalign_vision_process.py, videoalign_prompt_template.py).

VideoAlign scores a generated video against its caption with a Qwen2-VL backbone and a
linear Bradley–Terry head ``rm_head`` (hidden → ``output_dim``, no bias) read at one or more
token positions: the last real token, the mean over real tokens, or the three special
tokens ``<|VQ_reward|>``, ``<|MQ_reward|>``, ``<|TA_reward|>`` (visual quality, motion
quality, text alignment; with ``output_dim == 3`` token i contributes head output i).
Scores are optionally normalised with the checkpoint's ``inference_config`` means and
standard deviations, and ``Overall = VQ + MQ + TA``.

Checkpoint directory layout (the VideoAlign training code's, so released checkpoints load):
``model_config.json`` with ``data_config`` / ``model_config`` / ``peft_lora_config`` /
``inference_config``, and ``checkpoint-{step}/`` holding either a full ``model.pth`` or a
LoRA ``adapter_model.safetensors`` plus ``non_lora_state_dict.pth``.  LoRA factors are
merged into the base weights at load time (``W += s·B·A`` with ``s = α/r``, or ``α/√r``
with rsLoRA), so scoring runs on plain Linears; no PEFT/TRL dependency.

Differences from the reference, by design: frames are taken straight from the decoded
video tensor (the reference writes each video to a temporary mp4 and reads it back);
frame sampling and the Qwen-VL resize rule are reimplemented below.
"""
from __future__ import annotations

import glob
import json
import math
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

REWARD_TOKENS = ("<|VQ_reward|>", "<|MQ_reward|>", "<|TA_reward|>")
DIMENSIONS = ("VQ", "MQ", "TA")

# ---------------------------------------------------------------------------- prompts
# The scoring prompts are data of the checkpoint: the model was trained on exactly these
# texts, so they are kept word for word (VideoAlign's prompt_template.py).
_DIM_TEXT = {
    "VQ": ("visual quality", "the quality of the video in terms of clearness, resolution, brightness, and color"),
    "TA": ("text-to-video alignment", "the alignment between the text prompt and the video content and motion"),
    "MQ": ("motion quality", "the quality of the motion in terms of consistency, smoothness, and completeness"),
    "Overall": ("Overall Performance", "the overall performance of the video in terms of visual quality, "
                                       "text-to-video alignment, and motion quality"),
}

_TEMPLATES = {
    "simple": "\nPlease evaluate the {dimension_name} of a generated video. Consider {dimension_description}.\n"
              "The text prompt used for generation is \"{text_prompt}\".\n",
    "video_score": "\nSuppose you are an expert in judging and evaluating the quality of AI-generated videos,\n"
                   "please watch the frames of a given video and see the text prompt for generating the video,\n"
                   "then give scores based on its {dimension_name}, i.e., {dimension_description}.\n"
                   "Output a float number from 1.0 to 5.0 for this dimension,\n"
                   "the higher the number is, the better the video performs in that sub-score,\n"
                   "the lowest 1.0 means Bad, the highest 5.0 means Perfect/Real (the video is like a real video).\n"
                   "The text prompt used for generation is \"{text_prompt}\".\n",
}

_CRITERIA_HEAD = (
    "\nYou are tasked with evaluating a generated video based on three distinct criteria: Visual Quality, Motion "
    "Quality, and Text Alignment. Please provide a rating from 0 to 10 for each of the three categories, with 0 "
    "being the worst and 10 being the best. Each evaluation should be independent of the others.\n\n")
_VQ_BLOCK = (
    "**Visual Quality:**  \n"
    "Evaluate the overall visual quality of the video, with a focus on static factors. The following "
    "sub-dimensions should be considered:\n"
    "- **Reasonableness:** The video should not contain any significant biological or logical errors, such as "
    "abnormal body structures or nonsensical environmental setups.\n"
    "- **Clarity:** Evaluate the sharpness and visibility of the video. The image should be clear and easy to "
    "interpret, with no blurring or indistinct areas.\n"
    "- **Detail Richness:** Consider the level of detail in textures, materials, lighting, and other visual "
    "elements (e.g., hair, clothing, shadows).\n"
    "- **Aesthetic and Creativity:** Assess the artistic aspects of the video, including the color scheme, "
    "composition, atmosphere, depth of field, and the overall creative appeal. The scene should convey a sense "
    "of harmony and balance.\n"
    "- **Safety:** The video should not contain harmful or inappropriate content, such as political, violent, or "
    "adult material. If such content is present, the image quality and satisfaction score should be the lowest "
    "possible. \n\n")
_MQ_BLOCK = (
    "**Motion Quality:**  \n"
    "Assess the dynamic aspects of the video, with a focus on dynamic factors. Consider the following "
    "sub-dimensions:\n"
    "- **Stability:** Evaluate the continuity and stability between frames. There should be no sudden, unnatural "
    "jumps, and the video should maintain stable attributes (e.g., no fluctuating colors, textures, or missing "
    "body parts).\n"
    "- **Naturalness:** The movement should align with physical laws and be realistic. For example, clothing "
    "should flow naturally with motion, and facial expressions should change appropriately (e.g., blinking, "
    "mouth movements).\n"
    "- **Aesthetic Quality:** The movement should be smooth and fluid. The transitions between different motions "
    "or camera angles should be seamless, and the overall dynamic feel should be visually pleasing.\n"
    "- **Fusion:** Ensure that elements in motion (e.g., edges of the subject, hair, clothing) blend naturally "
    "with the background, without obvious artifacts or the feeling of cut-and-paste effects.\n"
    "- **Clarity of Motion:** The video should be clear and smooth in motion. Pay attention to any areas where "
    "the video might have blurry or unsteady sections that hinder visual continuity.\n"
    "- **Amplitude:** If the video is largely static or has little movement, assign a low score for motion "
    "quality.\n\n")
_TA_BLOCK = (
    "**Text Alignment:**  \n"
    "Assess how well the video matches the textual prompt across the following sub-dimensions:\n"
    "- **Subject Relevance** Evaluate how accurately the subject(s) in the video (e.g., person, animal, object) "
    "align with the textual description. The subject should match the description in terms of number, "
    "appearance, and behavior.\n"
    "- **Motion Relevance:** Evaluate if the dynamic actions (e.g., gestures, posture, facial expressions like "
    "talking or blinking) align with the described prompt. The motion should match the prompt in terms of type, "
    "scale, and direction.\n"
    "- **Environment Relevance:** Assess whether the background and scene fit the prompt. This includes checking "
    "if real-world locations or scenes are accurately represented, though some stylistic adaptation is "
    "acceptable.  \n"
    "- **Style Relevance:** If the prompt specifies a particular artistic or stylistic style, evaluate how well "
    "the video adheres to this style.\n"
    "- **Camera Movement Relevance:** Check if the camera movements (e.g., following the subject, focus shifts) "
    "are consistent with the expected behavior from the prompt.\n\n"
    "Textual prompt - {text_prompt}\n")


def _detailed(special: bool) -> str:
    if special:
        return (_CRITERIA_HEAD + _VQ_BLOCK.rstrip("\n") + "\n\nPlease provide the ratings of Visual Quality: "
                + REWARD_TOKENS[0] + "\nEND\n\n" + _MQ_BLOCK.rstrip("\n") + "\n\nPlease provide the ratings of "
                "Motion Quality: " + REWARD_TOKENS[1] + "\nEND\n\n" + _TA_BLOCK + "Please provide the ratings of "
                "Text Alignment: " + REWARD_TOKENS[2] + "\nEND\n")
    return (_CRITERIA_HEAD + _VQ_BLOCK + _MQ_BLOCK + "\n" + _TA_BLOCK
            + "Please provide the ratings of Visual Quality, Motion Quality, and Text Alignment.\n")


def build_prompt(caption: str, dimension, template_type: str) -> str:
    """Scoring prompt for ``caption`` (template types: none, simple, video_score, detailed,
    detailed_special)."""
    if template_type == "none":
        return caption
    if template_type in ("detailed", "detailed_special"):
        return _detailed(template_type == "detailed_special").format(text_prompt=caption)
    if template_type not in _TEMPLATES:
        raise ValueError(f"unknown VideoAlign prompt template {template_type!r}")
    dims = list(dimension) if isinstance(dimension, (list, tuple)) else [dimension]
    if len(dims) > 1:
        name = "overall performance(" + ", ".join(_DIM_TEXT[d][0] for d in dims) + ")"
        desc = "the overall performance of the video"
    else:
        name, desc = _DIM_TEXT[dims[0]]
    return _TEMPLATES[template_type].format(dimension_name=name, dimension_description=desc, text_prompt=caption)


# ---------------------------------------------------------------------------- frames
PATCH_FACTOR = 28                         # Qwen-VL: 14-pixel patches merged 2 × 2
FRAME_FACTOR = 2                          # frames are consumed in temporal pairs
VIDEO_MIN_PIXELS = 128 * 28 * 28
VIDEO_MAX_PIXELS = 768 * 28 * 28
VIDEO_TOTAL_PIXELS = 24576 * 28 * 28


def _round_to(x: float, f: int) -> int:
    return int(round(x / f)) * f


def vl_resize(height: int, width: int, factor: int = PATCH_FACTOR, min_pixels: int = VIDEO_MIN_PIXELS,
              max_pixels: int = VIDEO_MAX_PIXELS) -> Tuple[int, int]:
    """Target (h, w): multiples of ``factor`` near the input size, rescaled (keeping the
    aspect ratio) into [min_pixels, max_pixels] — the Qwen-VL resize rule."""
    if max(height, width) / min(height, width) > 200:
        raise ValueError("aspect ratio above 200")
    h = max(factor, _round_to(height, factor))
    w = max(factor, _round_to(width, factor))
    if h * w > max_pixels:
        s = math.sqrt(height * width / max_pixels)
        h = max(factor, math.floor(height / s / factor) * factor)
        w = max(factor, math.floor(width / s / factor) * factor)
    elif h * w < min_pixels:
        s = math.sqrt(min_pixels / (height * width))
        h = math.ceil(height * s / factor) * factor
        w = math.ceil(width * s / factor) * factor
    return h, w


def frame_indices(total: int, video_fps: float, nframes: Optional[int] = None, fps: Optional[float] = 2.0,
                  sample_type: str = "uniform", min_frames: int = 4, max_frames: int = 768) -> List[int]:
    """Frames to feed the model: ``nframes`` (rounded to pairs) or ``fps`` frames per second
    (clamped to [min_frames, max_frames], rounded to pairs), spread uniformly; or the
    ``multi_pts`` pattern (4 clusters of 6 consecutive frames of an 8-fps resampling)."""
    if sample_type == "multi_pts":
        per, pts, rate = 6, 4, 8
        n = int(total * rate // video_fps)
        grid = torch.linspace(0, total - 1, n).round().long().tolist()
        centers = torch.linspace(per // 2, n - per // 2 - 1, pts).round().long().tolist()
        return [i for c in centers for i in grid[c - per // 2:c + per // 2]]
    if sample_type != "uniform":
        raise ValueError(f"unknown frame sampling {sample_type!r}")
    if nframes is not None:
        n = _round_to(nframes, FRAME_FACTOR)
    else:
        lo = math.ceil(min_frames / FRAME_FACTOR) * FRAME_FACTOR
        hi = math.floor(min(max_frames, total) / FRAME_FACTOR) * FRAME_FACTOR
        n = _round_to(min(max(total / video_fps * fps, lo), hi), FRAME_FACTOR)
    n = min(n, total)
    if n < FRAME_FACTOR:
        raise ValueError(f"video of {total} frames is too short for VideoAlign")
    return torch.linspace(0, total - 1, n).round().long().tolist()


def prepare_frames(video: torch.Tensor, video_fps: float, nframes=None, fps=2.0, max_pixels=None,
                   sample_type="uniform") -> torch.Tensor:
    """uint8/float video [T, H, W, C] (0..255) → sampled, bicubic-resized float frames
    [T', C, h, w] (0..255) ready for the Qwen2-VL video processor."""
    v = torch.as_tensor(video)
    idx = frame_indices(v.shape[0], video_fps, nframes=nframes, fps=None if nframes is not None else fps,
                        sample_type=sample_type)
    v = v[idx].permute(0, 3, 1, 2).float()
    n, _, H, W = v.shape
    cap = max(min(VIDEO_MAX_PIXELS, VIDEO_TOTAL_PIXELS / n * FRAME_FACTOR), int(VIDEO_MIN_PIXELS * 1.05))
    h, w = vl_resize(H, W, max_pixels=max_pixels if max_pixels is not None else cap)
    v = F.interpolate(v, size=(h, w), mode="bicubic", align_corners=False, antialias=True)
    return v.clamp(0, 255)


# ---------------------------------------------------------------------------- config + weights
@dataclass
class VideoAlignConfig:
    model_name_or_path: str
    output_dim: int = 3
    reward_token: str = "special"
    use_special_tokens: bool = True
    eval_dim: object = "VQ"
    prompt_template_type: str = "detailed_special"
    fps: Optional[float] = 2.0
    num_frames: Optional[int] = None
    max_frame_pixels: int = 240 * 320
    sample_type: str = "uniform"
    lora_enable: bool = False
    lora_r: int = 16
    lora_alpha: int = 32
    use_rslora: bool = False
    norm: Dict[str, float] = field(default_factory=dict)

    @classmethod
    def from_dir(cls, path: str) -> "VideoAlignConfig":
        with open(os.path.join(path, "model_config.json")) as f:
            c = json.load(f)
        dc, mc, lc = c.get("data_config", {}), c.get("model_config", {}), c.get("peft_lora_config", {})
        return cls(model_name_or_path=mc["model_name_or_path"], output_dim=mc.get("output_dim", 3),
                   reward_token=mc.get("reward_token", "last"), use_special_tokens=mc.get("use_special_tokens", False),
                   eval_dim=dc.get("eval_dim", "VQ"), prompt_template_type=dc.get("prompt_template_type", "none"),
                   fps=dc.get("fps", 2.0), num_frames=dc.get("num_frames"),
                   max_frame_pixels=dc.get("max_frame_pixels", 240 * 320), sample_type=dc.get("sample_type", "uniform"),
                   lora_enable=lc.get("lora_enable", False), lora_r=lc.get("lora_r", 16),
                   lora_alpha=lc.get("lora_alpha", 32), use_rslora=lc.get("use_rslora", False),
                   norm=c.get("inference_config") or {})


def find_checkpoint(path: str, step: int = -1) -> str:
    """``checkpoint-{step}`` under ``path`` (the newest one when step is -1 or absent)."""
    cands = sorted(glob.glob(os.path.join(path, "checkpoint-*")), key=lambda p: int(p.rsplit("-", 1)[-1]))
    if not cands:
        raise FileNotFoundError(f"no checkpoint-* directory in {path}")
    if step is not None and step >= 0:
        want = os.path.join(path, f"checkpoint-{step}")
        if want in cands:
            return want
    return cands[-1]


def _canonical_key(k: str) -> str:
    """Training-time key (PEFT-wrapped, pre-5.x transformers layout) → this module's key."""
    for pre in ("base_model.model.", "module."):
        if k.startswith(pre):
            k = k[len(pre):]
    if k.startswith("model.") and not k.startswith(("model.language_model.", "model.visual.")):
        k = "model.language_model." + k[len("model."):]
    elif k.startswith("visual."):
        k = "model." + k
    return k


def merge_training_state(model_sd: Dict[str, torch.Tensor], tensors: Dict[str, torch.Tensor],
                         lora_scale: float) -> Dict[str, torch.Tensor]:
    """Fold a VideoAlign checkpoint (full weights and/or LoRA factors, training-time key
    names) into a state dict of :class:`VideoAlignRewardModel`; LoRA pairs
    ``X.lora_A[.default].weight`` / ``X.lora_B[.default].weight`` become ``X.weight += s·B·A``."""
    out = dict(model_sd)
    lora: Dict[str, Dict[str, torch.Tensor]] = {}
    for k, v in tensors.items():
        if ".lora_A." in k or ".lora_B." in k:
            base = k.split(".lora_")[0]
            lora.setdefault(_canonical_key(base), {})["A" if ".lora_A." in k else "B"] = v
            continue
        ck = _canonical_key(k).replace(".base_layer.", ".")
        if ck in out:
            out[ck] = v.to(out[ck].dtype)
    for base, ab in lora.items():
        wk = base + ".weight"
        if wk not in out or "A" not in ab or "B" not in ab:
            raise KeyError(f"LoRA factors for {base} do not match a weight of the model")
        w = out[wk].float() + lora_scale * (ab["B"].float() @ ab["A"].float())
        out[wk] = w.to(model_sd[wk].dtype)
    return out


class VideoAlignRewardModel(nn.Module):
    """Qwen2-VL backbone + ``rm_head``; ``forward`` returns pooled reward logits [B, n]."""

    def __init__(self, vl_model: nn.Module, output_dim: int = 3, reward_token: str = "special",
                 special_token_ids: Optional[Sequence[int]] = None, pad_token_id: Optional[int] = None):
        super().__init__()
        self.vl = vl_model
        cfg = vl_model.config
        hidden = getattr(getattr(cfg, "text_config", cfg), "hidden_size")
        self.rm_head = nn.Linear(hidden, output_dim, bias=False)
        self.output_dim = output_dim
        self.special_token_ids = list(special_token_ids) if special_token_ids else None
        self.reward_token = "special" if self.special_token_ids else reward_token
        self.pad_token_id = pad_token_id

    def state_dict_for_checkpoint(self) -> Dict[str, torch.Tensor]:
        sd = {k[len("vl."):]: v for k, v in self.state_dict().items() if k.startswith("vl.")}
        sd["rm_head.weight"] = self.rm_head.weight
        return sd

    def load_checkpoint_tensors(self, sd: Dict[str, torch.Tensor]) -> None:
        head = sd.pop("rm_head.weight", None)
        self.vl.load_state_dict(sd, strict=True)
        if head is not None:
            with torch.no_grad():
                self.rm_head.weight.copy_(head)

    def forward(self, input_ids, attention_mask=None, pixel_values_videos=None, video_grid_thw=None, **kw):
        h = self.vl.model(input_ids=input_ids, attention_mask=attention_mask,
                          pixel_values_videos=pixel_values_videos, video_grid_thw=video_grid_thw,
                          **kw).last_hidden_state
        logits = self.rm_head(h)                                    # [B, L, out]
        B = input_ids.shape[0]
        if self.reward_token == "special":
            sel = torch.zeros_like(input_ids, dtype=torch.bool)
            for tid in self.special_token_ids:
                sel |= input_ids == tid
            pooled = logits[sel].view(B, len(self.special_token_ids), -1)
            if self.output_dim == len(self.special_token_ids):
                pooled = pooled.diagonal(dim1=1, dim2=2)           # token i → head output i
            return pooled.reshape(B, -1)
        # index of the last real token: right padding ends at the first pad token
        if self.pad_token_id is None:
            last = torch.full((B,), input_ids.shape[1] - 1, device=input_ids.device)
        else:
            last = (torch.eq(input_ids, self.pad_token_id).int().argmax(-1) - 1) % input_ids.shape[1]
        if self.reward_token == "last":
            return logits[torch.arange(B, device=logits.device), last]
        if self.reward_token == "mean":
            return torch.stack([logits[i, :max(int(last[i]), 1)].mean(0) for i in range(B)])
        raise ValueError(f"unknown reward token mode {self.reward_token!r}")


class VideoAlignScorer:
    """Scores decoded videos with a VideoAlign checkpoint directory (see module docstring)."""

    def __init__(self, device, load_from_pretrained: Optional[str], load_from_pretrained_step: int = -1,
                 reward_dim: str = "Overall", use_norm: bool = True, num_frames=None, fps=None, max_pixels=None,
                 dtype=torch.bfloat16, save_fps: float = 8.0, processor=None, vl_model=None):
        if not load_from_pretrained or not os.path.isdir(load_from_pretrained):
            raise FileNotFoundError("VideoAlign needs `load_from_pretrained` pointing at its checkpoint directory")
        self.cfg = VideoAlignConfig.from_dir(load_from_pretrained)
        self.device = device
        self.reward_dim = reward_dim
        self.use_norm = use_norm
        self.num_frames = num_frames if num_frames is not None else self.cfg.num_frames
        self.fps = fps if fps is not None else self.cfg.fps
        self.max_pixels = max_pixels if max_pixels is not None else self.cfg.max_frame_pixels
        self.video_fps = save_fps           # frame rate the decoded videos are taken to have
        if processor is None:
            from transformers import AutoProcessor
            processor = AutoProcessor.from_pretrained(self.cfg.model_name_or_path, padding_side="right")
        self.processor = processor
        special = None
        if self.cfg.use_special_tokens:
            processor.tokenizer.add_special_tokens({"additional_special_tokens": list(REWARD_TOKENS)})
            special = processor.tokenizer.convert_tokens_to_ids(list(REWARD_TOKENS))
        if vl_model is None:
            from transformers import Qwen2VLForConditionalGeneration
            vl_model = Qwen2VLForConditionalGeneration.from_pretrained(self.cfg.model_name_or_path,
                                                                        torch_dtype=torch.float32)
        if special is not None:
            vl_model.resize_token_embeddings(len(processor.tokenizer))
        model = VideoAlignRewardModel(vl_model, self.cfg.output_dim, self.cfg.reward_token, special,
                                      processor.tokenizer.pad_token_id)
        ck = find_checkpoint(load_from_pretrained, load_from_pretrained_step)
        full = os.path.join(ck, "model.pth")
        if os.path.exists(full):
            tensors = torch.load(full, map_location="cpu", weights_only=True)
        else:
            from safetensors.torch import load_file
            tensors = dict(torch.load(os.path.join(ck, "non_lora_state_dict.pth"), map_location="cpu",
                                      weights_only=True))
            tensors.update(load_file(os.path.join(ck, "adapter_model.safetensors")))
        r, a = self.cfg.lora_r, self.cfg.lora_alpha
        scale = a / math.sqrt(r) if self.cfg.use_rslora else a / r
        model.load_checkpoint_tensors(merge_training_state(model.state_dict_for_checkpoint(), tensors, scale))
        self.model = model.to(device=device, dtype=dtype).eval()

    def normalise(self, scores: Dict[str, float]) -> Dict[str, float]:
        if self.use_norm and self.cfg.norm:
            scores = {d: (scores[d] - self.cfg.norm[f"{d}_mean"]) / self.cfg.norm[f"{d}_std"] for d in DIMENSIONS}
        scores = dict(scores)
        scores["Overall"] = scores["VQ"] + scores["MQ"] + scores["TA"]
        return scores

    @torch.no_grad()
    def score(self, videos: Sequence[torch.Tensor], prompts: Sequence[str]) -> List[Dict[str, float]]:
        """videos: [T, H, W, C] uint8 (or float 0..255) each; returns VQ/MQ/TA/Overall per video."""
        frames = [prepare_frames(v, self.video_fps, nframes=self.num_frames, fps=self.fps,
                                 max_pixels=self.max_pixels, sample_type=self.cfg.sample_type) for v in videos]
        convs = [[{"role": "user", "content": [
            {"type": "video"},
            {"type": "text", "text": build_prompt(p, self.cfg.eval_dim, self.cfg.prompt_template_type)}]}]
            for p in prompts]
        texts = [self.processor.apply_chat_template(c, tokenize=False, add_generation_prompt=True) for c in convs]
        batch = self.processor(text=texts, videos=frames, padding=True, return_tensors="pt",
                               videos_kwargs={"do_rescale": True})
        batch = {k: (v.to(self.device) if torch.is_tensor(v) else v) for k, v in batch.items()}
        if "pixel_values_videos" in batch:
            batch["pixel_values_videos"] = batch["pixel_values_videos"].to(next(self.model.parameters()).dtype)
        logits = self.model(**batch).float().cpu()
        return [self.normalise({d: float(r[i]) for i, d in enumerate(DIMENSIONS)}) for r in logits]

    def __call__(self, videos, prompts) -> List[float]:
        vids = [torch.as_tensor(v) for v in videos]
        return [s[self.reward_dim] for s in self.score(vids, prompts)]
